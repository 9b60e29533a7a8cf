"""ctypes binding of libqwen3_5_cuda.so (the cs1_* ABI, include/qwen3_5_ops.h).

Arguments that are device pointers accept an int address or any object with a
`data_ptr()` method (a torch tensor); `stream` accepts an int / cudaStream_t
address, None (the legacy default stream) or an object with `cuda_stream`.
Every call that returns a status raises `Cs1Error` on a nonzero code, the way
the reference's loader maps codes to errors (cuda.rs:707-717).
"""
import ctypes
import os

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
P = ctypes.c_void_p
I = ctypes.c_int
Z = ctypes.c_size_t
F = ctypes.c_float
U32 = ctypes.c_uint32
U64 = ctypes.c_uint64

# name: (restype, [argtypes]) -- mirrors include/qwen3_5_ops.h
SIGNATURES = {
    "cs1_abi_version": (U32, []),
    "cs1_error_string": (ctypes.c_char_p, [I]),
    "cs1_set_device": (I, [I]),
    "cs1_get_device": (I, [P]),
    "cs1_bf16_finite": (I, [P, Z, P, P]),
    "cs1_malloc": (I, [P, Z]),
    "cs1_free": (I, [P]),
    "cs1_stream_create": (I, [P]),
    "cs1_stream_sync": (I, [P]),
    "cs1_stream_destroy": (I, [P]),
    "cs1_graph_begin": (I, [P]),
    "cs1_graph_end": (I, [P, P]),
    "cs1_graph_launch": (I, [P, P]),
    "cs1_graph_destroy": (I, [P]),
    "cs1_upload": (I, [P, P, Z, P]),
    "cs1_download": (I, [P, P, Z, P]),
    "cs1_copy_dd": (I, [P, P, Z, P]),
    "cs1_copy2d": (I, [P, Z, P, Z, Z, Z, P]),
    "cs1_fault_status": (U32, [I]),
    "cs1_wait_selftest": (I, [ctypes.c_longlong, P]),
    "cs1_embed": (I, [P, P, P, I, I, P]),
    "cs1_rms_norm": (I, [P, P, P, I, I, F, P]),
    "cs1_add_rms_norm": (I, [P, P, P, P, I, I, F, P]),
    "cs1_gated_rms_norm": (I, [P, P, I, P, P, I, I, I, F, P]),
    "cs1_gdn_conv": (I, [P, I, P, P, P, P, I, I, I, P]),
    "cs1_gdn_conv_vector": (I, [P, I, P, P, P, P, I, I, I, P]),
    "cs1_gdn_conv_prefix": (I, [P, P, I, P, P, P, P, I, I, I, P]),
    "cs1_gdn_conv_batch": (I, [P, P, I, P, P, P, P, P, Z, I, I, P]),
    "cs1_attention_gated_shared": (I, [P, P, P, I, P, P, P, P, I, I, I, I, I, F, P]),
    "cs1_attention_gated_shared_batch": (I, [P, P, P, I, P, P, P, P, P, Z, I, I, I, I, F, P]),
    "cs1_attention_gated_batch": (I, [P, P, P, I, P, P, P, Z, I, I, I, F, P]),
    "cs1_gdn_gates": (I, [P, P, I, P, P, P, P, I, I, P]),
    "cs1_gdn_batch_workspace_floats": (Z, [I, I, I]),
    "cs1_gdn_prefill_batch": (I, [P, P, P, P, P, P, P, Z, P, Z, I, I, F, P]),
    "cs1_gdn_prefill_batch_shared": (I, [P, P, P, P, P, P, P, Z, P, Z, I, I, F, P, P]),
    "cs1_gdn_workspace_floats": (Z, [I, I]),
    "cs1_gdn_fp32_create": (P, [Z]),
    "cs1_gdn_fp32_destroy": (None, [P]),
    "cs1_gdn_fp32_workspace_floats": (Z, [I, I]),
    "cs1_gdn_prefill_fp32": (I, [P, P, P, P, P, P, P, P, I, I, I, F, P]),
    "cs1_gdn_prefill_fp32_x": (I, [P, P, P, P, P, P, P, P, I, I, I, F, P, P, P]),
    "cs1_gdn_prefill": (I, [P, P, P, P, P, P, P, I, I, I, F, P]),
    "cs1_gdn_prefill_wide": (I, [P, P, P, P, P, P, P, I, I, I, F, P]),
    "cs1_gdn_prefill_noalloc": (I, [P, P, P, P, P, P, I, I, I, F, P]),
    "cs1_gdn_prefill_x": (I, [P, P, P, P, P, P, P, I, I, I, F, P, P, P]),
    "cs1_gdn_prefill_batch_x": (I, [P, P, P, P, P, P, P, Z, P, Z, I, I, F, P, I, P, P]),
    "cs1_attn_prep": (I, [P, P, I, P, P, P, P, P, P, P, I, I, I, I, I, F, P]),
    "cs1_attention": (I, [P, P, P, I, P, I, I, I, I, F, P]),
    "cs1_attention_gated": (I, [P, P, P, I, P, P, I, I, I, I, F, P]),
    "cs1_attention_gated_bidirectional": (I, [P, P, P, I, P, P, I, I, I, I, F, P]),
    "cs1_attention_gated_prefix_bidirectional": (I, [P, P, P, I, P, P, I, I, I, I, I, F, P]),
    "cs1_attention_gated_prefix": (I, [P, P, P, I, P, P, I, I, I, I, F, I, P]),
    "cs1_sigmoid_gate": (I, [P, P, Z, P]),
    "cs1_silu_mul": (I, [P, I, P, I, I, P]),
    "cs1_gemm_create": (P, [Z]),
    "cs1_gemm_create_fixed": (P, [Z, I]),
    "cs1_gemm_create_matched": (P, [Z, I]),
    "cs1_gemm_compatible": (I, [P, P, I, I, I]),
    "cs1_gemm_destroy": (None, [P]),
    "cs1_gemm_enable_equivalent_tiles": (I, [P]),
    "cs1_gemm": (I, [P, P, P, P, I, I, I, I, P]),
    "cs1_gemm_packed": (I, [P, P, P, P, P, Z, I, I, P]),
    "cs1_gemm_reuse_check": (I, [P, P, Z, P, Z, I, I]),
    "cs1_gemm_reuse": (I, [P, P, P, P, I, I, I, I, P]),
    "cs1_gemm_residual": (I, [P, P, P, P, I, I, I, I, P]),
    "cs1_gemm_swiglu": (I, [P, P, P, P, I, I, I, I, P]),
    "cs1_head_score": (I, [P, I, P, I, P, P, I, I, P, P]),
    "cs1_batch_desc_bytes": (Z, []),
    "cs1_batch_desc_pack": (I, [P, Z, P, Z]),
    "cs1_embed_dyn": (I, [P, P, P, I, I, P, P]),
    "cs1_clear_tail_dyn": (I, [P, Z, Z, I, I, P, P]),
    "cs1_rms_norm_dyn": (I, [P, P, P, I, I, F, P, P]),
    "cs1_add_rms_norm_dyn": (I, [P, P, P, P, I, I, F, P, P]),
    "cs1_gated_rms_norm_dyn": (I, [P, P, I, P, P, I, I, I, F, P, P]),
    "cs1_gemm_dyn": (I, [P, P, P, P, I, I, I, I, I, P, P]),
    "cs1_gdn_conv_dyn": (I, [P, P, I, P, P, P, P, I, I, I, I, P, P]),
    "cs1_gdn_gates_dyn": (I, [P, P, I, P, P, P, P, I, I, P, P]),
    "cs1_gdn_prefill_dyn": (I, [P, P, P, P, P, P, P, P, I, I, I, I, F, P, I, P, P, P]),
    "cs1_gdn_front_dyn": (I, [P, P, I, P, P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, P, P]),
    "cs1_gdn_front_batch": (I, [P, P, I, P, P, P, P, P, P, P, P, P, P, P, P, I, P, Z, I, I, P]),
    "cs1_gdn_prefill_batch_xn": (I, [P, P, P, P, P, P, P, P, P, Z, I, I, F, P, I, P, P]),
    "cs1_attn_prep_dyn": (I, [P, P, I, P, P, P, P, P, P, P, I, I, I, I, I, F, P, P]),
    "cs1_attention_dyn": (I, [P, P, P, I, P, P, P, P, I, I, I, I, I, I, F, P, P]),
    "cs1_head_score_dyn": (I, [P, I, P, I, P, P, I, I, P, P, P]),
    "cs1_fill_random": (I, [P, Z, I, U64, F, F, I, P]),
    "cs1_vision_linear": (I, [P, P, P, P, P, I, I, I, P]),
    "cs1_gemm_f32": (I, [P, P, P, P, I, I, I, P]),
    "cs1_vision_norm": (I, [P, P, P, P, I, I, P]),
    "cs1_vision_position": (I, [P, P, P, P, I, P]),
    "cs1_vision_rope": (I, [P, P, P, P, P, I, P]),
    "cs1_vision_attention": (I, [P, P, P, P, I, P]),
    "cs1_vision_bias": (I, [P, P, Z, I, P]),
    "cs1_vision_gelu": (I, [P, Z, I, P]),
    "cs1_vision_add": (I, [P, P, Z, P]),
    "cs1_vision_to_float": (I, [P, P, Z, P]),
    "cs1_vision_lora_add": (I, [P, P, Z, F, P]),
}

# Functions whose int return is a size or a boolean-like status, not an error code.
_NOT_STATUS = {"cs1_gemm_compatible", "cs1_gemm_enable_equivalent_tiles", "cs1_gemm_reuse_check"}


def lib_path(name="libqwen3_5_cuda.so"):
    return os.path.join(_PKG, "lib", name)


class Cs1Error(RuntimeError):
    def __init__(self, name, code, text):
        super().__init__(f"{name} failed with {code}: {text}")
        self.code = code


def _arg(x):
    if x is None:
        return None
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if hasattr(x, "cuda_stream"):
        return x.cuda_stream
    return x


class Cs1:
    """The cs1_* library. `Cs1().cs1_gemm(...)` raises on a nonzero status;
    `Cs1().raw.cs1_gemm(...)` returns the code."""

    def __init__(self, path=None):
        path = path or lib_path()
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is missing: run system1-omni_b200/build.py")
        self.path = path
        self.raw = ctypes.CDLL(path)
        self.missing = set()
        for name, (res, args) in SIGNATURES.items():
            try:
                fn = getattr(self.raw, name)
            except AttributeError:  # optional / additive symbol absent from this library
                self.missing.add(name)
                continue
            fn.restype = res
            fn.argtypes = args

    def __getattr__(self, name):
        if name not in SIGNATURES or name in self.__dict__.get("missing", ()):
            raise AttributeError(name)
        fn = getattr(self.raw, name)
        res = SIGNATURES[name][0]

        def call(*args):
            r = fn(*[_arg(a) for a in args])
            if res is I and name not in _NOT_STATUS and r != 0:
                raise Cs1Error(name, r, self.raw.cs1_error_string(r).decode())
            return r

        return call
