"""ctypes binding of liboasis_b200.so (declarations mirror include/oasis_b200.h).

This is the only route to compute: there is no CPU or PyTorch fallback. If the
shared library is missing, every entry point raises OasisLibraryError.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboasis_b200.so")

OASIS_DIT_SUBBLOCKS = 32
OASIS_ADALN_WIDTH = 6144
OASIS_VAE_BLOCKS = 12
OASIS_VAE_ENC_K = 1216

ERRORS = {
    -1: "OASIS_ERR_INVALID_ARG",
    -2: "OASIS_ERR_CUDA",
    -3: "OASIS_ERR_WORKSPACE",
    -4: "OASIS_ERR_DEVICE_TIMEOUT",
    -5: "OASIS_ERR_UNSUPPORTED",
}

vp = C.c_void_p
fp = C.c_void_p  # float* (device)


class OasisLibraryError(RuntimeError):
    """The CUDA library is not built or could not be loaded."""


class OasisError(RuntimeError):
    """A library call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed: {ERRORS.get(code, code)}: {msg}")
        self.code = code


class OasisDitSubBlock(C.Structure):
    _fields_ = [("qkv_w", vp), ("out_w", vp), ("out_b", fp), ("fc1_w", vp), ("fc1_b", fp),
                ("fc2_w", vp), ("fc2_b", fp)]


class OasisDitWeights(C.Structure):
    _fields_ = [("num_subblocks", C.c_int), ("sub", OasisDitSubBlock * OASIS_DIT_SUBBLOCKS),
                ("adaln_w", vp), ("adaln_b", fp), ("final_w", vp), ("final_b", fp),
                ("embed_w", fp), ("embed_b", fp), ("rope_spatial", fp), ("rope_temporal", fp)]


class OasisCondWeights(C.Structure):
    _fields_ = [("t_freqs", fp), ("t_w0", fp), ("t_b0", fp), ("t_w2", fp), ("t_b2", fp), ("ext_w", fp),
                ("ext_b", fp)]


class OasisVaeBlock(C.Structure):
    _fields_ = [("norm1_w", fp), ("norm1_b", fp), ("qkv_w", vp), ("qkv_b", fp), ("proj_w", vp),
                ("proj_b", fp), ("norm2_w", fp), ("norm2_b", fp), ("fc1_w", vp), ("fc1_b", fp),
                ("fc2_w", vp), ("fc2_b", fp)]


class OasisVaeWeights(C.Structure):
    _fields_ = [("post_quant_w", fp), ("post_quant_b", fp), ("num_blocks", C.c_int),
                ("blk", OasisVaeBlock * OASIS_VAE_BLOCKS), ("norm_w", fp), ("norm_b", fp),
                ("pred_w", vp), ("pred_b", fp), ("rope", fp)]


class OasisDitArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("frames", C.c_int), ("z", fp), ("cond", fp), ("v_out", fp),
                ("last_frame_only", C.c_int), ("workspace", vp), ("workspace_bytes", C.c_size_t)]


class OasisDdimCoeffs(C.Structure):
    _fields_ = [("at_sqrt", C.c_float), ("one_minus_at_sqrt", C.c_float), ("inv_at_sqrt", C.c_float),
                ("inv_sigma", C.c_float), ("an_sqrt", C.c_float), ("one_minus_an_sqrt", C.c_float)]


class OasisStepArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("frames", C.c_int), ("chunk", fp), ("context_z", fp), ("cond", fp),
                ("coeffs", OasisDdimCoeffs), ("workspace", vp), ("workspace_bytes", C.c_size_t)]


class OasisVaeArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("latent", fp), ("image", fp), ("workspace", vp),
                ("workspace_bytes", C.c_size_t)]


class OasisVaeEncoderWeights(C.Structure):
    _fields_ = [("patch_w", vp), ("patch_b", fp), ("num_blocks", C.c_int),
                ("blk", OasisVaeBlock * OASIS_VAE_BLOCKS), ("norm_w", fp), ("norm_b", fp),
                ("quant_w", vp), ("quant_b", fp), ("rope", fp)]


class OasisVaeEncodeArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("image", fp), ("latent", fp), ("chunk", fp), ("workspace", vp),
                ("workspace_bytes", C.c_size_t)]


class OasisFrameArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("frames", C.c_int), ("steps", C.c_int), ("chunk", fp), ("context_z", fp),
                ("cond", fp), ("coeffs", C.POINTER(OasisDdimCoeffs)), ("image", fp), ("skip_decode", C.c_int),
                ("workspace", vp), ("workspace_bytes", C.c_size_t)]


class OasisGemmArgs(C.Structure):
    _fields_ = [("a", vp), ("lda", C.c_longlong), ("w", vp), ("m", C.c_int), ("n", C.c_int), ("k", C.c_int),
                ("mode", C.c_int), ("out", vp), ("ldo", C.c_longlong), ("bias", fp), ("resid", fp),
                ("ldr", C.c_longlong), ("gate", fp), ("ldg", C.c_longlong), ("rows_per_frame", C.c_int),
                ("rope", fp), ("rope_div", C.c_int), ("rope_mod", C.c_int), ("block_n", C.c_int),
                ("splits", C.c_int), ("workspace", vp), ("workspace_bytes", C.c_size_t), ("rope_dim", C.c_int),
                ("rope_stride", C.c_int), ("ln_out", vp), ("ln_mod", fp), ("ln_ld_mod", C.c_longlong),
                ("ln_shift_off", C.c_longlong), ("ln_scale_off", C.c_longlong), ("ln_eps", C.c_float)]


# int (*)(float* buf, size_t count, void* user, cudaStream_t stream)
ALLREDUCE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p)


class OasisTpArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("frames", C.c_int), ("heads", C.c_int), ("z", fp), ("cond", fp),
                ("v_out", fp), ("partial", fp), ("allreduce", ALLREDUCE_FN), ("allreduce_user", vp),
                ("workspace", vp), ("workspace_bytes", C.c_size_t)]


COLLECTIVE_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_int, C.c_void_p, C.c_void_p)
OASIS_DTYPE_F32 = 0
OASIS_DTYPE_BF16 = 1
OASIS_IPC_HANDLE_BYTES = 64


class OasisTpSpArgs(C.Structure):
    _fields_ = [("batch", C.c_int), ("frames", C.c_int), ("heads", C.c_int), ("rank", C.c_int), ("world", C.c_int),
                ("z", fp), ("cond", fp), ("v_out", fp), ("partial_dtype", C.c_int), ("partial", vp), ("shard", vp),
                ("xn_local", vp), ("xn", vp), ("v_local", fp), ("reduce_scatter", COLLECTIVE_FN),
                ("all_gather", COLLECTIVE_FN), ("user", vp), ("workspace", vp), ("workspace_bytes", C.c_size_t),
                ("comm_stream", vp), ("chunks", C.c_int), ("reserve_sms", C.c_int)]


class OasisLayerNormArgs(C.Structure):
    _fields_ = [("x", fp), ("y", vp), ("rows_out", C.c_int), ("P", C.c_int), ("in_group", C.c_longlong),
                ("in_off", C.c_longlong), ("frame_mul", C.c_longlong), ("frame_add", C.c_longlong),
                ("eps", C.c_float), ("mod", fp), ("ld_mod", C.c_longlong), ("shift_off", C.c_longlong),
                ("scale_off", C.c_longlong), ("affine_w", fp), ("affine_b", fp)]


# name -> (restype, argtypes). Every symbol the header declares.
SIGNATURES = {
    "oasis_last_error": (C.c_char_p, []),
    "oasis_get_last_error": (C.c_char_p, []),
    "oasis_device_error": (C.c_int, [C.c_int]),
    "oasis_version": (C.c_char_p, []),
    "oasis_launch_count": (C.c_ulonglong, []),
    "oasis_dit_workspace_size": (C.c_size_t, [C.c_int, C.c_int]),
    "oasis_dit_forward": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisDitArgs), vp]),
    "oasis_ddim_update": (C.c_int, [fp, fp, C.POINTER(OasisDdimCoeffs), C.c_longlong, vp]),
    "oasis_step_workspace_size": (C.c_size_t, [C.c_int, C.c_int]),
    "oasis_ddim_step": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisStepArgs), vp]),
    "oasis_patch_embed": (C.c_int, [C.POINTER(OasisDitWeights), fp, C.c_int, fp, C.c_longlong, C.c_longlong, vp]),
    "oasis_bridge_unpatchify": (C.c_int, [fp, fp, C.c_int, vp]),
    "oasis_vae_workspace_size": (C.c_size_t, [C.c_int]),
    "oasis_vae_decode": (C.c_int, [C.POINTER(OasisVaeWeights), C.POINTER(OasisVaeArgs), vp]),
    "oasis_vae_encoder_workspace_size": (C.c_size_t, [C.c_int]),
    "oasis_vae_encode": (C.c_int, [C.POINTER(OasisVaeEncoderWeights), C.POINTER(OasisVaeEncodeArgs), vp]),
    "oasis_frame_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "oasis_generate_frame": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisVaeWeights),
                                       C.POINTER(OasisFrameArgs), vp]),
    "oasis_tp_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "oasis_dit_forward_tp": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisTpArgs), vp]),
    "oasis_cond_workspace_size": (C.c_size_t, [C.c_int]),
    "oasis_compute_cond": (C.c_int, [C.POINTER(OasisCondWeights), fp, C.c_int, fp, C.c_int, fp, vp, C.c_size_t, vp]),
    "oasis_tp_sp_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int]),
    "oasis_dit_forward_tp_sp": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisTpSpArgs), vp]),
    "oasis_peer_alloc": (C.c_int, [C.c_size_t, C.POINTER(vp)]),
    "oasis_peer_free": (C.c_int, [vp]),
    "oasis_ipc_get_handle": (C.c_int, [vp, vp]),
    "oasis_ipc_open_handle": (C.c_int, [vp, C.POINTER(vp)]),
    "oasis_ipc_close_handle": (C.c_int, [vp]),
    "oasis_peer_copy": (C.c_int, [vp, vp, C.c_size_t, vp]),
    "oasis_peer_signal": (C.c_int, [vp, C.c_int, vp]),
    "oasis_peer_wait": (C.c_int, [vp, C.c_int, C.c_int, C.c_int, C.c_longlong, vp]),
    "oasis_reduce_slots": (C.c_int, [vp, vp, C.c_longlong, vp, C.c_int, C.c_int, C.c_longlong, C.c_int, vp]),
    "oasis_kv_cache_size": (C.c_size_t, [C.c_int, C.c_int]),
    "oasis_dit_precompute_past": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisDitArgs), vp, C.c_size_t, vp]),
    "oasis_dit_forward_current": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisDitArgs), vp, C.c_size_t,
                                            C.c_int, vp]),
    "oasis_frame_kv_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "oasis_generate_frame_kv": (C.c_int, [C.POINTER(OasisDitWeights), C.POINTER(OasisVaeWeights),
                                          C.POINTER(OasisFrameArgs), vp]),
    "oasis_gemm": (C.c_int, [C.POINTER(OasisGemmArgs), vp]),
    "oasis_gemm_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
    "oasis_gemm_plan": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_int),
                                  C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_size_t)]),
    "oasis_gemm_static_scratch": (C.c_int, [C.POINTER(OasisGemmArgs), vp]),
    "oasis_gemm_static_scratch_capacity": (C.c_size_t, []),
    "oasis_layernorm": (C.c_int, [C.POINTER(OasisLayerNormArgs), vp]),
    "oasis_silu_bf16": (C.c_int, [fp, vp, C.c_longlong, vp]),
    "oasis_attention_spatial": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp]),
    "oasis_attention_tc": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp]),
    "oasis_attention_temporal": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp]),
    "oasis_attention_temporal_cached": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp]),
    "oasis_gated_residual": (C.c_int, [fp, fp, fp, fp, C.c_longlong, C.c_int, C.c_int, vp]),
    "oasis_post_quant": (C.c_int, [fp, fp, fp, fp, C.c_int, vp]),
}

_lib = None


def load() -> C.CDLL:
    """Loads liboasis_b200.so (once) and declares every exported function."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise OasisLibraryError(
            f"{LIB_PATH} is missing: build it with __graft_entry__.build() (nvcc, sm_100a). "
            "There is no CPU fallback.")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        f = getattr(lib, name)
        f.restype = res
        f.argtypes = args
    _lib = lib
    return lib


def call(name: str, *args) -> int:
    """Calls an int-returning entry point; raises OasisError on a non-zero status."""
    lib = load()
    rc = getattr(lib, name)(*args)
    if rc != 0:
        raise OasisError(name, rc, lib.oasis_last_error().decode(errors="replace"))
    return rc


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (None for None)."""
    return None if t is None else t.data_ptr()
