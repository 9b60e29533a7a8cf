// A loopback stand-in for the few NCCL calls the context-parallel prefill makes
// (ncclGetUniqueId, ncclCommInitRank, ncclCommDestroy, ncclSend, ncclRecv, ncclAllGather,
// ncclGroupStart / ncclGroupEnd, ncclGetErrorString), for ranks that are threads of one
// process on ONE GPU. Test infrastructure: it lets the host's context-parallel path
// (piece agreement, per-layer state / conv history / K,V hand-off) run where only one GPU
// exists. Transfers are stream-ordered device-to-device copies:
//   - a send publishes (source, bytes, an event recorded on the sender's stream) in the
//     (sender, receiver) FIFO;
//   - the matching receive makes the receiver's stream wait for that event, copies, and
//     records a completion event, which the sender's stream then waits for, so the sender
//     does not overwrite its source before the copy has read it (NCCL's rendezvous);
//   - inside a group, sends are published first and receives run before the sends wait,
//     so the rank chain 0 -> 1 -> ... -> n-1 cannot deadlock.
// No kernel of this library waits on anything; every host wait gives up after a limit
// (LOOPBACK_NCCL_TIMEOUT_S, default 120 s) and returns ncclSystemError.
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <vector>

namespace {

struct Message {
    const void* src = nullptr;
    size_t bytes = 0;
    cudaEvent_t ready = nullptr;  // recorded on the sender's stream after the send was posted
    cudaEvent_t done = nullptr;   // recorded on the receiver's stream after the copy
    bool taken = false;
};

struct Group {
    int world = 0;
    int joined = 0;
    std::mutex mu;
    std::condition_variable cv;
    std::map<std::pair<int, int>, std::deque<std::shared_ptr<Message>>> fifo;  // (from, to)
    // all-gather rendezvous: a reusable barrier (generation, arrivals), per-rank source and events
    long gen = 0;
    int posted = 0;
    std::vector<const void*> ag_src;
    std::vector<cudaEvent_t> ag_ready, ag_done;
};

struct Comm {
    std::shared_ptr<Group> group;
    int rank = 0;
};

struct PendingOp {
    bool send;
    void* buf;
    size_t bytes;
    int peer;
    Comm* comm;
    cudaStream_t stream;
};

std::mutex g_mu;
std::map<unsigned long long, std::shared_ptr<Group>> g_groups;
thread_local int t_depth = 0;
thread_local std::vector<PendingOp> t_ops;

std::chrono::seconds limit() {
    const char* s = std::getenv("LOOPBACK_NCCL_TIMEOUT_S");
    const int v = s ? std::atoi(s) : 0;
    return std::chrono::seconds(v > 0 ? v : 120);
}

size_t type_size(ncclDataType_t t) {
    switch (t) {
        case ncclInt8: case ncclUint8: return 1;
        case ncclFloat16: case ncclBfloat16: return 2;
        case ncclInt32: case ncclUint32: case ncclFloat32: return 4;
        case ncclInt64: case ncclUint64: case ncclFloat64: return 8;
        default: return 0;
    }
}

cudaEvent_t record(cudaStream_t s) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    if (cudaEventRecord(e, s) != cudaSuccess) {
        cudaEventDestroy(e);
        return nullptr;
    }
    return e;
}

// Runs the queued operations of one group (or one lone call).
ncclResult_t run(std::vector<PendingOp>& ops) {
    std::vector<std::shared_ptr<Message>> sent;
    std::vector<PendingOp*> sends;
    for (auto& op : ops) {
        if (!op.send) continue;
        auto msg = std::make_shared<Message>();
        msg->src = op.buf;
        msg->bytes = op.bytes;
        msg->ready = record(op.stream);
        if (!msg->ready) return ncclUnhandledCudaError;
        Group& g = *op.comm->group;
        {
            std::lock_guard<std::mutex> lk(g.mu);
            g.fifo[{op.comm->rank, op.peer}].push_back(msg);
        }
        g.cv.notify_all();
        sent.push_back(msg);
        sends.push_back(&op);
    }
    for (auto& op : ops) {
        if (op.send) continue;
        Group& g = *op.comm->group;
        std::shared_ptr<Message> msg;
        {
            std::unique_lock<std::mutex> lk(g.mu);
            auto& q = g.fifo[{op.peer, op.comm->rank}];
            if (!g.cv.wait_for(lk, limit(), [&] { return !q.empty(); })) return ncclSystemError;
            msg = q.front();
            q.pop_front();
        }
        if (msg->bytes != op.bytes) return ncclInvalidUsage;
        if (cudaStreamWaitEvent(op.stream, msg->ready, 0) != cudaSuccess) return ncclUnhandledCudaError;
        if (op.bytes && cudaMemcpyAsync(op.buf, msg->src, op.bytes, cudaMemcpyDeviceToDevice, op.stream) != cudaSuccess)
            return ncclUnhandledCudaError;
        cudaEvent_t done = record(op.stream);
        if (!done) return ncclUnhandledCudaError;
        {
            std::lock_guard<std::mutex> lk(g.mu);
            msg->done = done;
            msg->taken = true;
        }
        g.cv.notify_all();
    }
    for (size_t i = 0; i < sent.size(); i++) {
        Group& g = *sends[i]->comm->group;
        auto& msg = sent[i];
        {
            std::unique_lock<std::mutex> lk(g.mu);
            if (!g.cv.wait_for(lk, limit(), [&] { return msg->taken; })) return ncclSystemError;
        }
        if (cudaStreamWaitEvent(sends[i]->stream, msg->done, 0) != cudaSuccess) return ncclUnhandledCudaError;
        cudaEventDestroy(msg->ready);
        cudaEventDestroy(msg->done);
    }
    return ncclSuccess;
}

ncclResult_t enqueue(PendingOp op) {
    if (!op.comm || op.peer < 0 || op.peer >= op.comm->group->world || op.peer == op.comm->rank)
        return ncclInvalidArgument;
    t_ops.push_back(op);
    if (t_depth > 0) return ncclSuccess;
    std::vector<PendingOp> ops;
    ops.swap(t_ops);
    return run(ops);
}

}  // namespace

extern "C" {

ncclResult_t ncclGetUniqueId(ncclUniqueId* id) {
    if (!id) return ncclInvalidArgument;
    static std::mutex mu;
    static unsigned long long next = 1;
    std::lock_guard<std::mutex> lk(mu);
    std::memset(id, 0, sizeof(*id));
    const unsigned long long key = next++;
    std::memcpy(id->internal, &key, sizeof(key));
    return ncclSuccess;
}

ncclResult_t ncclCommInitRank(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank) {
    if (!comm || nranks < 1 || rank < 0 || rank >= nranks) return ncclInvalidArgument;
    unsigned long long key;
    std::memcpy(&key, id.internal, sizeof(key));
    std::shared_ptr<Group> g;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto& slot = g_groups[key];
        if (!slot) {
            slot = std::make_shared<Group>();
            slot->world = nranks;
            slot->ag_src.assign(nranks, nullptr);
            slot->ag_ready.assign(nranks, nullptr);
            slot->ag_done.assign(nranks, nullptr);
        }
        if (slot->world != nranks) return ncclInvalidUsage;
        g = slot;
        g->joined++;
    }
    auto* c = new Comm;
    c->group = g;
    c->rank = rank;
    *comm = reinterpret_cast<ncclComm_t>(c);
    return ncclSuccess;
}

ncclResult_t ncclCommDestroy(ncclComm_t comm) {
    delete reinterpret_cast<Comm*>(comm);
    return ncclSuccess;
}

ncclResult_t ncclGroupStart() {
    t_depth++;
    return ncclSuccess;
}

ncclResult_t ncclGroupEnd() {
    if (t_depth <= 0) return ncclInvalidUsage;
    if (--t_depth > 0) return ncclSuccess;
    std::vector<PendingOp> ops;
    ops.swap(t_ops);
    return run(ops);
}

ncclResult_t ncclSend(const void* buf, size_t count, ncclDataType_t t, int peer, ncclComm_t comm,
                      cudaStream_t stream) {
    return enqueue({true, const_cast<void*>(buf), count * type_size(t), peer, reinterpret_cast<Comm*>(comm), stream});
}

ncclResult_t ncclRecv(void* buf, size_t count, ncclDataType_t t, int peer, ncclComm_t comm, cudaStream_t stream) {
    return enqueue({false, buf, count * type_size(t), peer, reinterpret_cast<Comm*>(comm), stream});
}

// Every rank's `count` elements, in rank order, into every rank's recv buffer. Three
// bounded host barriers: all sources posted; every rank's reads enqueued (on its own
// stream, after the sources' ready events); every rank's stream made to wait for all
// reads, so no source is overwritten before every rank has copied it.
ncclResult_t ncclAllGather(const void* send, void* recv, size_t count, ncclDataType_t t, ncclComm_t comm,
                           cudaStream_t stream) {
    auto* c = reinterpret_cast<Comm*>(comm);
    if (!c || t_depth > 0) return ncclInvalidUsage;
    Group& g = *c->group;
    const size_t bytes = count * type_size(t);
    std::unique_lock<std::mutex> lk(g.mu);
    auto barrier = [&]() {
        const long gen = g.gen;
        if (++g.posted == g.world) {
            g.posted = 0;
            g.gen++;
            g.cv.notify_all();
            return true;
        }
        return g.cv.wait_for(lk, limit(), [&] { return g.gen != gen; });
    };
    cudaEvent_t ready = record(stream);
    if (!ready) return ncclUnhandledCudaError;
    g.ag_src[c->rank] = send;
    g.ag_ready[c->rank] = ready;
    if (!barrier()) return ncclSystemError;
    for (int r = 0; r < g.world; r++) {
        if (cudaStreamWaitEvent(stream, g.ag_ready[r], 0) != cudaSuccess) return ncclUnhandledCudaError;
        if (bytes && cudaMemcpyAsync(static_cast<char*>(recv) + r * bytes, g.ag_src[r], bytes,
                                     cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
            return ncclUnhandledCudaError;
    }
    cudaEvent_t done = record(stream);
    if (!done) return ncclUnhandledCudaError;
    g.ag_done[c->rank] = done;
    if (!barrier()) return ncclSystemError;
    for (int r = 0; r < g.world; r++)
        if (cudaStreamWaitEvent(stream, g.ag_done[r], 0) != cudaSuccess) return ncclUnhandledCudaError;
    if (!barrier()) return ncclSystemError;
    cudaEventDestroy(ready);
    cudaEventDestroy(done);
    return ncclSuccess;
}

const char* ncclGetErrorString(ncclResult_t r) {
    switch (r) {
        case ncclSuccess: return "no error";
        case ncclUnhandledCudaError: return "loopback: CUDA call failed";
        case ncclSystemError: return "loopback: a peer did not arrive within the time limit";
        case ncclInvalidArgument: return "loopback: invalid argument";
        case ncclInvalidUsage: return "loopback: invalid usage (mismatched sizes or ranks)";
        default: return "loopback: error";
    }
}

}  // extern "C"
