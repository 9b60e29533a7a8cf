"""Python bindings of the B200 Qwen3.5 hybrid decision-model prefill.

Thin ctypes layer over the two native libraries built in-tree by
`system1-omni_b200/build.py`:

* `libqwen3_5_cuda.so` -- the cs1_* C ABI (include/qwen3_5_ops.h): every
  operation of the prefill as a hand-written sm_100a kernel.
* `libs1_model.so`     -- the C++ prefill host (include/s1_model.h): weights,
  packed / shared-prefix forward, scorer head, CUDA graphs; and the worker-side
  request processing (include/s1_processing.h): tokenizer, request contract,
  calibrated responses.

There is no fallback: a missing library raises at import of the binding.
"""
from .cs1 import Cs1, Cs1Error, lib_path
from .dispatch import dispatch, request_cost, shard
from .model import (Config, Model, checkpoint_check, checkpoint_list, config_from_hf, cp_agree, cp_piece_status,
                    cp_pieces, cp_unique_id, pack_ranges, preset, shared_prefix)
from .processing import Processor, Tokenizer

__all__ = ["Cs1", "Cs1Error", "lib_path", "Config", "Model", "checkpoint_check", "checkpoint_list", "config_from_hf",
           "cp_agree", "cp_piece_status", "cp_pieces", "cp_unique_id", "dispatch", "pack_ranges", "preset",
           "request_cost", "shard", "shared_prefix", "Processor", "Tokenizer"]
