"""ctypes binding of libs1_model.so (include/s1_model.h): the decision-model prefill.

`Model` mirrors the reference worker's executor interface: load weights, run a
packed-candidate prefill, score each candidate's final token with the learned
head (src/models/open_jev/native/src/executor.rs:237-343 for the call pattern).
"""
import ctypes
from dataclasses import dataclass, field

import numpy as np

from .cs1 import lib_path

P = ctypes.c_void_p
I = ctypes.c_int
Z = ctypes.c_size_t


class _Cfg(ctypes.Structure):
    _fields_ = [("hidden", I), ("intermediate", I), ("n_layers", I), ("layer_types", ctypes.POINTER(I)),
                ("lin_k_heads", I), ("lin_v_heads", I), ("lin_k_dim", I), ("lin_v_dim", I), ("heads", I),
                ("kv_heads", I), ("head_dim", I), ("rotary_half", I), ("theta", ctypes.c_double),
                ("eps", ctypes.c_float), ("vocab", I), ("labels", I)]


@dataclass
class Config:
    """Qwen3.5 hybrid scorer shape (Transformers Qwen3_5TextConfig fields, renamed)."""
    hidden: int
    intermediate: int
    layer_types: list            # "gdn" / "attn" per layer
    lin_k_heads: int
    lin_v_heads: int
    heads: int
    kv_heads: int
    vocab: int
    labels: int = 8
    lin_k_dim: int = 128
    lin_v_dim: int = 128
    head_dim: int = 256
    rotary_half: int = 32
    theta: float = 1.0e7
    eps: float = 1e-6
    name: str = field(default="custom")

    def weight_count(self):
        H, I_ = self.hidden, self.intermediate
        kd, vd, hv = self.lin_k_heads * 128, self.lin_v_heads * 128, self.lin_v_heads
        n = self.vocab * H + H + self.labels * (H + 1)
        for t in self.layer_types:
            n += 2 * H + 3 * H * I_
            if t == "gdn":
                conv = 2 * kd + vd
                n += (conv + vd + 2 * hv) * H + conv * 4 + 2 * hv + 128 + H * vd
            else:
                n += (2 * self.heads * 256 + 2 * self.kv_heads * 256) * H + 512 + H * self.heads * 256
        return n

    def projection_flops_per_token(self):
        """2 * sum(N * K) over every projection (the tensor-core work per token)."""
        H, I_ = self.hidden, self.intermediate
        kd, vd, hv = self.lin_k_heads * 128, self.lin_v_heads * 128, self.lin_v_heads
        f = 0
        for t in self.layer_types:
            f += 3 * H * I_
            if t == "gdn":
                f += (2 * kd + vd + vd + 2 * hv) * H + H * vd
            else:
                f += (2 * self.heads * 256 + 2 * self.kv_heads * 256) * H + H * self.heads * 256
        return 2 * f


def _hybrid(n, interval=4):
    return ["attn" if (i + 1) % interval == 0 else "gdn" for i in range(n)]


def preset(name):
    """The benchmark shapes (4B, 9B, 27B) and small test shapes."""
    table = {
        "4b": (2560, 9216, 32, 16, 32, 16, 4, 151936),
        "9b": (4096, 12288, 32, 16, 32, 16, 4, 151936),
        "27b": (5120, 17408, 64, 16, 48, 24, 4, 151936),
        "tiny": (256, 512, 4, 2, 4, 4, 2, 512),
        "tiny8": (512, 1024, 8, 2, 6, 6, 2, 1024),
    }
    H, I_, L, hk, hv, hq, hkv, vocab = table[name]
    return Config(H, I_, _hybrid(L), hk, hv, hq, hkv, vocab, name=name)


def _lib():
    lib = ctypes.CDLL(lib_path("libs1_model.so"))
    lib.s1_model_create.restype = P
    lib.s1_model_create.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Cfg), I, I, I]
    lib.s1_model_destroy.argtypes = [P]
    lib.s1_model_destroy.restype = None
    lib.s1_model_error.restype = ctypes.c_char_p
    lib.s1_model_error.argtypes = [P]
    lib.s1_model_set_weight.argtypes = [P, ctypes.c_char_p, P, Z]
    lib.s1_model_get_weight.argtypes = [P, ctypes.c_char_p, P, Z]
    lib.s1_model_init_random.argtypes = [P, ctypes.c_uint64, ctypes.c_float]
    lib.s1_model_forward.argtypes = [P, P, P, Z, P, P]
    lib.s1_model_forward_shared.argtypes = [P, P, Z, P, P, Z, P, P]
    lib.s1_model_run_layers.argtypes = [P, P, P, Z, I, I, P]
    lib.s1_model_stage.argtypes = [P, P, P, Z]
    lib.s1_model_run_staged.argtypes = [P]
    lib.s1_model_fetch_logits.argtypes = [P, P]
    lib.s1_model_set_graphs.argtypes = [P, I]
    lib.s1_model_set_dynamic.argtypes = [P, I]
    lib.s1_model_graph_count.argtypes = [P]
    lib.s1_model_stream.restype = P
    lib.s1_model_stream.argtypes = [P]
    lib.s1_model_last_launches.restype = ctypes.c_long
    lib.s1_model_last_launches.argtypes = [P]
    lib.s1_model_fused.argtypes = [P]
    lib.s1_config_from_hf.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Cfg), P, I]
    lib.s1_model_load_checkpoint.argtypes = [P, ctypes.c_char_p]
    lib.s1_model_load_head.argtypes = [P, ctypes.c_char_p, I, I]
    lib.s1_checkpoint_list.restype = ctypes.c_long
    lib.s1_checkpoint_list.argtypes = [ctypes.c_char_p, P, Z]
    lib.s1_cp_unique_id.argtypes = [ctypes.c_char_p, P]
    lib.s1_model_cp_init.argtypes = [P, ctypes.c_char_p, P, I, I]
    lib.s1_model_forward_cp.argtypes = [P, P, Z, Z, P, P]
    lib.s1_checkpoint_check.argtypes = [ctypes.c_char_p, ctypes.POINTER(_Cfg)]
    lib.s1_model_get_config.argtypes = [P, ctypes.POINTER(_Cfg)]
    lib.s1_checkpoint_error.restype = ctypes.c_char_p
    lib.s1_checkpoint_error.argtypes = []
    lib.s1_cp_piece_status.argtypes = [P, Z, Z, I, I, I, Z]
    lib.s1_cp_agree.argtypes = [P, I, ctypes.c_char_p, Z]
    lib.s1_pack_ranges.argtypes = [P, Z, Z, Z, P]
    lib.s1_shared_prefix.restype = Z
    lib.s1_shared_prefix.argtypes = [P, P, Z, Z]
    return lib


_LIB = None


def _get():
    global _LIB
    if _LIB is None:
        import os
        path = lib_path("libs1_model.so")
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing: run system1-omni_b200/build.py")
        _LIB = _lib()
    return _LIB


def pack_ranges(lengths, max_sequences=16, max_tokens=4096):
    """[(start, end)] launch ranges (open_jev batching.rs:9-25), computed by the C++ host."""
    lib = _get()
    n = len(lengths)
    arr = np.asarray(lengths, dtype=np.uintp)
    starts = np.zeros(n + 1, dtype=np.uintp)
    r = lib.s1_pack_ranges(arr.ctypes.data, n, max_sequences, max_tokens, starts.ctypes.data)
    if r < 0:
        raise ValueError("invalid packing arguments")
    return [(int(starts[i]), int(starts[i + 1])) for i in range(r)]


def shared_prefix(inputs, minimum=2049):
    """Aligned shared prefix of 2..16 candidates (batching.rs:29-49), computed by the C++ host."""
    lib = _get()
    arrays = [np.ascontiguousarray(x, dtype=np.int32) for x in inputs]
    ptrs = (ctypes.c_void_p * max(1, len(arrays)))(*[a.ctypes.data for a in arrays])
    lens = np.asarray([len(a) for a in arrays], dtype=np.uintp)
    return int(lib.s1_shared_prefix(ctypes.cast(ptrs, P), lens.ctypes.data, len(arrays), minimum))


def config_from_hf(config_json, labels=1, name="checkpoint"):
    """The Config of a Hugging Face Qwen3.5 config.json (or its text_config), read by the
    C++ host (model.rs:96-226 of the reference). labels: rows of the scorer head."""
    lib = _get()
    types = (I * 4096)()
    c = _Cfg()
    if lib.s1_config_from_hf(str(config_json).encode(), ctypes.byref(c), ctypes.cast(types, P), 4096) != 0:
        raise ValueError("config.json: " + lib.s1_checkpoint_error().decode())
    return Config(c.hidden, c.intermediate, ["gdn" if types[i] == 0 else "attn" for i in range(c.n_layers)],
                  c.lin_k_heads, c.lin_v_heads, c.heads, c.kv_heads, c.vocab, labels=labels, lin_k_dim=c.lin_k_dim,
                  lin_v_dim=c.lin_v_dim, head_dim=c.head_dim, rotary_half=c.rotary_half, theta=c.theta, eps=c.eps,
                  name=name)


def checkpoint_list(folder):
    """[(name, hf_name, dtype, shape)] of the language-model tensors of a checkpoint folder."""
    lib = _get()
    n = lib.s1_checkpoint_list(str(folder).encode(), None, 0)
    if n < 0:
        raise ValueError("checkpoint: " + lib.s1_checkpoint_error().decode())
    buf = ctypes.create_string_buffer(n)
    lib.s1_checkpoint_list(str(folder).encode(), buf, n)
    out = []
    for line in buf.value.decode().splitlines():
        name, hf, dtype, shape = line.split(" ")
        out.append((name, hf, dtype, tuple(int(x) for x in shape.split("x"))))
    return out


def checkpoint_check(folder, cfg):
    """Check a checkpoint folder against a Config (tensor set, shapes, dtypes, sizes) on
    the host, as Model.load_checkpoint does before it reads any payload. Raises ValueError."""
    lib = _get()
    types = (I * len(cfg.layer_types))(*[0 if t == "gdn" else 1 for t in cfg.layer_types])
    c = _Cfg(cfg.hidden, cfg.intermediate, len(cfg.layer_types), types, cfg.lin_k_heads, cfg.lin_v_heads,
             cfg.lin_k_dim, cfg.lin_v_dim, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.rotary_half,
             float(cfg.theta), float(cfg.eps), cfg.vocab, cfg.labels)
    if lib.s1_checkpoint_check(str(folder).encode(), ctypes.byref(c)) != 0:
        raise ValueError("checkpoint: " + lib.s1_checkpoint_error().decode())


def cp_pieces(cfg, tokens, world, align=64):
    """Piece lengths of a context-parallel split of one `tokens`-long prompt over `world`
    ranks (in prompt order), on `align`-token boundaries, sized so that every rank's
    estimated work is about the same: projection FLOPs in proportion to its tokens plus
    causal attention FLOPs in proportion to its queries times the keys they see (all
    earlier pieces and half of its own). The last rank takes the remainder."""
    lin = cfg.projection_flops_per_token()
    att = 4.0 * cfg.heads * cfg.head_dim * sum(1 for t in cfg.layer_types if t != "gdn")

    def cost(start, n):
        return lin * n + att * n * (start + n / 2.0)

    total = cost(0, tokens)
    lengths, start = [], 0
    for r in range(world - 1):
        left = world - r
        target = cost(start, tokens - start) / left if r else total / world
        lo, hi = 0, tokens - start
        while lo < hi:  # largest aligned n with cost(start, n) <= target
            mid = (lo + hi + 1) // 2
            if cost(start, mid) <= target:
                lo = mid
            else:
                hi = mid - 1
        down = lo // align * align  # the aligned length whose cost is nearer the target
        up = min(down + align, tokens - start - align)
        n = up if up > down and abs(cost(start, up) - target) < abs(cost(start, down) - target) else down
        n = max(align, n)
        lengths.append(n)
        start += n
    lengths.append(tokens - start)
    if lengths[-1] < align:
        raise ValueError("prompt too short for this many pieces")
    return lengths


def cp_piece_status(ids, start, rank, world, vocab, cap_tokens):
    """The checks forward_cp makes on one rank's piece (host only): 0 or a negative code."""
    a = np.ascontiguousarray(ids, np.int32)
    return int(_get().s1_cp_piece_status(a.ctypes.data if len(a) else None, len(a), start, rank, world, vocab,
                                         cap_tokens))


def cp_agree(table):
    """The verdict every rank reaches on all ranks' (status, start, len, 0) rows before a
    context-parallel forward: (0, "") or (-1, reason)."""
    t = np.ascontiguousarray(table, np.int64).reshape(-1, 4)
    msg = ctypes.create_string_buffer(256)
    rc = _get().s1_cp_agree(t.ctypes.data, len(t), msg, 256)
    return int(rc), msg.value.decode()


def cp_unique_id(nccl_library=None):
    """The 128-byte NCCL id of a context-parallel group, made on one rank and handed to
    every rank (for instance with torch.distributed.broadcast_object_list)."""
    lib = _get()
    buf = ctypes.create_string_buffer(128)
    if lib.s1_cp_unique_id((nccl_library or "").encode(), buf) != 0:
        raise RuntimeError("s1_cp_unique_id: " + lib.s1_model_error(None).decode())
    return buf.raw


class Model:
    """A prefill model on one GPU: `Model(cfg, device, max_tokens, max_seqs)`."""

    def __init__(self, cfg, device=0, max_tokens=4096, max_seqs=64, cs1_library=None):
        self.cfg = cfg
        self._lib = _get()
        self._types = (I * len(cfg.layer_types))(*[0 if t == "gdn" else 1 for t in cfg.layer_types])
        c = _Cfg(cfg.hidden, cfg.intermediate, len(cfg.layer_types), self._types, cfg.lin_k_heads, cfg.lin_v_heads,
                 cfg.lin_k_dim, cfg.lin_v_dim, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.rotary_half,
                 float(cfg.theta), float(cfg.eps), cfg.vocab, cfg.labels)
        path = (cs1_library or lib_path()).encode()
        self._h = self._lib.s1_model_create(path, ctypes.byref(c), device, max_tokens, max_seqs)
        if not self._h:
            raise RuntimeError("s1_model_create: " + self._lib.s1_model_error(None).decode())
        self.max_tokens, self.max_seqs = max_tokens, max_seqs

    def _check(self, rc, what):
        if rc != 0:
            raise RuntimeError(f"{what}: " + self._lib.s1_model_error(self._h).decode())

    def close(self):
        if getattr(self, "_h", None):
            self._lib.s1_model_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def set_weight(self, name, array):
        """array: numpy float32 holding bf16 values (converted here), or float32 for the head."""
        a = np.ascontiguousarray(array, dtype=np.float32)
        if name in ("head_w", "head_b"):
            data = a
        else:
            u = a.view(np.uint32).astype(np.uint64)
            data = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
        self._check(self._lib.s1_model_set_weight(self._h, name.encode(), data.ctypes.data, data.nbytes), name)

    def get_weight(self, name, shape):
        """Read a parameter back as float32 (bf16 values; float32 for the head)."""
        if name in ("head_w", "head_b"):
            out = np.zeros(shape, np.float32)
        else:
            out = np.zeros(shape, np.uint16)
        self._check(self._lib.s1_model_get_weight(self._h, name.encode(), out.ctypes.data, out.nbytes), name)
        if out.dtype == np.uint16:
            out = (out.astype(np.uint32) << 16).view(np.float32)
        return out

    def load(self, weights):
        for name, arr in weights.items():
            self.set_weight(name, arr)

    def load_checkpoint(self, folder):
        """Every language-model weight of a Hugging Face Qwen3.5 checkpoint folder."""
        if self._lib.s1_model_load_checkpoint(self._h, str(folder).encode()) != 0:
            raise RuntimeError("load_checkpoint: " + self._lib.s1_checkpoint_error().decode())

    def load_head(self, manifest_json):
        """The scorer head of an export manifest (open_jev_export.json)."""
        if self._lib.s1_model_load_head(self._h, str(manifest_json).encode(), self.cfg.labels, self.cfg.hidden) != 0:
            raise RuntimeError("load_head: " + self._lib.s1_checkpoint_error().decode())

    def cp_init(self, rank, world, uid, nccl_library=None):
        """Join a context-parallel group of `world` processes (one per GPU) as `rank`."""
        self._check(self._lib.s1_model_cp_init(self._h, (nccl_library or "").encode(), ctypes.c_char_p(uid), rank,
                                               world), "cp_init")
        self._cp_last = rank == world - 1

    def forward_cp(self, ids, start, hidden=False):
        """This rank's piece of one prompt (positions from `start`): logits [labels] (and the
        last hidden row) on the last rank, None on the others."""
        a = np.ascontiguousarray(ids, np.int32)
        logits = np.zeros(self.cfg.labels, np.float32)
        hid = np.zeros(self.cfg.hidden, np.float32) if hidden else None
        self._check(self._lib.s1_model_forward_cp(self._h, a.ctypes.data, len(a), start, logits.ctypes.data,
                                                  hid.ctypes.data if hidden else None), "forward_cp")
        if not getattr(self, "_cp_last", False):
            return (None, None) if hidden else None
        return (logits, hid) if hidden else logits

    def init_random(self, seed=0, std=0.02):
        self._check(self._lib.s1_model_init_random(self._h, seed, std), "init_random")

    def forward(self, seqs, hidden=False):
        """Packed candidates (list of int arrays) -> logits [n, labels] (and last hidden rows)."""
        ids = np.concatenate([np.asarray(s, np.int32) for s in seqs])
        lens = np.asarray([len(s) for s in seqs], dtype=np.uintp)
        logits = np.zeros((len(seqs), self.cfg.labels), np.float32)
        hid = np.zeros((len(seqs), self.cfg.hidden), np.float32) if hidden else None
        self._check(self._lib.s1_model_forward(self._h, ids.ctypes.data, lens.ctypes.data, len(seqs),
                                               logits.ctypes.data, hid.ctypes.data if hidden else None), "forward")
        return (logits, hid) if hidden else logits

    def forward_shared(self, prefix, suffixes, hidden=False):
        pre = np.asarray(prefix, np.int32)
        ids = np.concatenate([np.asarray(s, np.int32) for s in suffixes])
        lens = np.asarray([len(s) for s in suffixes], dtype=np.uintp)
        logits = np.zeros((len(suffixes), self.cfg.labels), np.float32)
        hid = np.zeros((len(suffixes), self.cfg.hidden), np.float32) if hidden else None
        self._check(self._lib.s1_model_forward_shared(self._h, pre.ctypes.data, len(pre), ids.ctypes.data,
                                                      lens.ctypes.data, len(suffixes), logits.ctypes.data,
                                                      hid.ctypes.data if hidden else None), "forward_shared")
        return (logits, hid) if hidden else logits

    def run_layers(self, seqs, first, last, residual):
        """Layers [first, last) of packed candidates from a residual stream (bf16 bit
        patterns, uint16 [sum lengths, H], the stream entering layer `first`); returns the
        stream leaving layer last - 1 in the same form."""
        ids = np.concatenate([np.asarray(s, np.int32) for s in seqs])
        lens = np.asarray([len(s) for s in seqs], dtype=np.uintp)
        res = np.ascontiguousarray(residual, dtype=np.uint16).copy()
        if res.shape != (len(ids), self.cfg.hidden):
            raise ValueError(f"residual must be [{len(ids)}, {self.cfg.hidden}] bf16 bits")
        self._check(self._lib.s1_model_run_layers(self._h, ids.ctypes.data, lens.ctypes.data, len(seqs), first, last,
                                                  res.ctypes.data), "run_layers")
        return res

    def stage(self, seqs):
        ids = np.concatenate([np.asarray(s, np.int32) for s in seqs])
        lens = np.asarray([len(s) for s in seqs], dtype=np.uintp)
        self._check(self._lib.s1_model_stage(self._h, ids.ctypes.data, lens.ctypes.data, len(seqs)), "stage")
        self._staged_n = len(seqs)  # a refused batch leaves the previous one staged

    def run_staged(self):
        self._check(self._lib.s1_model_run_staged(self._h), "run_staged")

    def fetch_logits(self):
        out = np.zeros((self._staged_n, self.cfg.labels), np.float32)
        self._check(self._lib.s1_model_fetch_logits(self._h, out.ctypes.data), "fetch_logits")
        return out

    def set_graphs(self, on):
        self._check(self._lib.s1_model_set_graphs(self._h, 1 if on else 0), "set_graphs")

    def set_dynamic(self, on):
        """Device-side batching: launches sized for capacities, the batch read from a device
        descriptor, so one captured graph serves every length vector of its capacities."""
        self._check(self._lib.s1_model_set_dynamic(self._h, 1 if on else 0), "set_dynamic")

    @property
    def graph_count(self):
        return int(self._lib.s1_model_graph_count(self._h))

    @property
    def stream(self):
        return self._lib.s1_model_stream(self._h)

    @property
    def last_launches(self):
        return int(self._lib.s1_model_last_launches(self._h))

    @property
    def fused(self):
        return bool(self._lib.s1_model_fused(self._h))
