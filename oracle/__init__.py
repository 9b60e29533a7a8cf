"""CPU oracle for the Qwen3.5 hybrid decision-model prefill.

TEST INFRASTRUCTURE ONLY. Nothing in the product path imports this package:
only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of
`bench.py` use it, and there only as the checker (or, for the CPU baseline,
as the timed CPU restatement of the reference's path).

It restates, in numpy, the arithmetic of the reference's CUDA backend
(`src/backends/cuda/qwen3_5/*.cu` of InferMatrixLab/system1-omni) and of the
Rust layer loop that drives it (`src/models/qwen3_5/native/src/model.rs`),
whose own parity anchor is Transformers' PyTorch Qwen3.5 code
(`transformers/models/qwen3_5/modeling_qwen3_5.py`, pinned by the reference at
5.17.0; this container has 5.5.0). The restatement is pinned against golden
vectors produced by that Transformers code (`tests/golden/make_golden.py`).

Modules:
  bf16     -- round-to-nearest-even bfloat16 helpers
  ops      -- one function per `cs1_*` operation (norms, conv, gates, prep, attention, GEMM)
  gdn      -- chunked Gated DeltaNet (fp32 and bf16-intermediate forms) and the float64 recurrence
  packing  -- candidate packing ranges, shared-prefix detection, positions, rotary tables
  model    -- configurations, seeded weights, the whole forward and the scorer head
"""
