"""ctypes binding of ``libmrsa_b200.so`` (the C ABI declared in ``include/mrsa.h``).

The library is loaded once, in-tree.  There is no fallback: if it is missing
or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes as C
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmrsa_b200.so")

ERR_NULL, ERR_SHAPE, ERR_ALIGN, ERR_LAUNCH, ERR_ARG, ERR_WORKSPACE = -1, -2, -3, -4, -5, -6
BF16, F32 = 0, 1
WEIGHTS_AFFINE, WEIGHTS_SOFTMAX = 0, 1
GEMM_PLAIN, GEMM_SWIGLU, GEMM_RESIDUAL = 0, 1, 2

_vp, _i64, _f32, _int, _sz = C.c_void_p, C.c_int64, C.c_float, C.c_int, C.c_size_t

# name -> argtypes (restype int unless listed in _RESTYPE)
_SIGS = {
    "mrsa_strerror": [_int],
    "mrsa_last_error": [],
    "mrsa_abi_version": [],
    "mrsa_yarn_inv_freq": [_int, C.c_double, C.c_double, _int, C.c_double, C.c_double, _int, _vp, _vp],
    "mrsa_rope": [_vp, _vp, _i64, _vp, _vp, _i64, _vp, _vp, _f32, _vp, _vp, _int, _i64, _i64, _i64, _vp],
    "mrsa_qcal_route_query": [_vp, _vp, _vp, _vp, _vp, _f32, _f32, _vp, _vp, _f32, _vp,
                              _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_chunk_pool": [_vp, _i64, _i64, _vp, _vp, _f32, _vp, _vp, _vp, _vp, _vp,
                        _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_remote_drop_mask": [_vp, _vp, _i64, _i64, _i64, _i64, _vp],
    "mrsa_remote_drop_mask_positions": [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_route_topk": [_vp, _vp, _int, _vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _int, _vp, _vp,
                        _int, _f32, _f32, _f32, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz,
                        _vp],
    "mrsa_route_topk_workspace_size": [_i64, _i64, _i64, _i64, _i64, _int],
    "mrsa_route_weights": [_vp, _vp, _vp, _vp, _vp, _vp, _int, _f32, _f32, _f32,
                           _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_local_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _i64, _f32,
                             _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_local_attention_f16v": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _i64, _f32,
                                  _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_selected_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f32, _int,
                                _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_selected_attention_f16v": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f32, _int,
                                _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_local_attention_positions": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _i64, _f32,
                                       _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_flex_attention": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _i64, _f32,
                            _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_candidate_token_scores": [_vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _i64, _i64, _i64,
                                    _i64, _i64, _vp],
    "mrsa_selected_token_attention": [_vp, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _i64, _i64,
                                      _i64, _i64, _vp],
    "mrsa_selected_token_attention_smem": [_i64, _i64],
    "mrsa_selected_attention_keep": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f32, _int, _int,
                                     _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_convert_bf16_to_f16": [_vp, _vp, _i64, _vp],
    "mrsa_fuse_outputs": [_vp, _vp, _vp, _vp, _i64, _i64, _vp],
    "mrsa_probe_tile_gather": [_vp, _vp, _vp, _i64, _i64, _i64, _int, _i64, _vp, _vp],
    "mrsa_selected_attention_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _f32, _int,
                                         _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _vp, _sz, _vp],
    "mrsa_selected_attention_backward_workspace": [_i64, _i64, _i64, _i64, _i64],
    "mrsa_chunk_pool_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_route_weights_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _f32, _f32, _f32,
                                    _i64, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_route_scores_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _f32, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                   _vp, _sz, _vp],
    "mrsa_route_scores_backward_workspace": [_i64, _i64, _i64, _i64, _i64],
    "mrsa_fuse_outputs_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _vp],
    "mrsa_gemm_bf16": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp],
    "mrsa_rms_norm": [_vp, _vp, _vp, _i64, _i64, _f32, _vp],
    "mrsa_local_attention_backward": [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz, _i64, _int,
                                      _i64, _f32, _i64, _i64, _i64, _i64, _i64, _vp],
    "mrsa_local_attention_backward_workspace": [_i64, _i64, _i64],
    "mrsa_device_error_flags": [_int],
    "mrsa_wait_selftest": [_vp, _int, _vp],
    "mrsa_route_layer_workspace_size": [_vp],
    "mrsa_route_layer_forward": [_vp, _vp, _sz, _vp],
    "mrsa_route_layer_forward_noalloc": [_vp, _vp],
}
_RESTYPE = {"mrsa_strerror": C.c_char_p, "mrsa_last_error": C.c_char_p, "mrsa_route_layer_workspace_size": _sz,
            "mrsa_route_topk_workspace_size": _sz, "mrsa_selected_token_attention_smem": _sz,
            "mrsa_selected_attention_backward_workspace": _sz, "mrsa_route_scores_backward_workspace": _sz,
            "mrsa_local_attention_backward_workspace": _sz}

EXPORTED = tuple(_SIGS)

_lib = None


def load():
    """Load the library (idempotent).  Raises if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                "(the MRSA ops have no CPU fallback)")
        lib = C.CDLL(LIB_PATH)
        for name, argtypes in _SIGS.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPE.get(name, _int)
        _lib = lib
    return _lib


class MRSAError(RuntimeError):
    pass


def check(rc: int, what: str):
    if rc == 0:
        return
    msg = load().mrsa_strerror(rc).decode()
    if rc in (ERR_SHAPE, ERR_ARG, ERR_NULL, ERR_ALIGN):
        raise ValueError(f"{what}: {msg} (code {rc})")
    if rc == ERR_LAUNCH:
        msg += f" [{load().mrsa_last_error().decode()}]"
    raise MRSAError(f"{what}: {msg} (code {rc})")


def ptr(t: torch.Tensor | None):
    return None if t is None else C.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return C.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def call(name: str, *args):
    check(getattr(load(), name)(*args), name)


class RouteLayerArgs(C.Structure):
    """``mrsa_route_layer_args`` of ``include/mrsa.h``."""

    _fields_ = [
        ("q_pre", _vp), ("k_pre", _vp), ("v", _vp), ("hidden", _vp), ("position_ids", _vp),
        ("key_valid", _vp), ("inv_freq", _vp), ("w_in", _vp), ("w_out", _vp),
        ("norm_weight", _vp), ("bias_scale", _vp), ("out", _vp),
        ("attention_factor", _f32), ("rms_eps", _f32), ("qcal_scale", _f32),
        ("temperature", _f32), ("gate_scale", _f32), ("gate_offset", _f32),
        ("batch", _i64), ("seq_len", _i64), ("q_heads", _i64), ("kv_heads", _i64),
        ("head_dim", _i64), ("hidden_size", _i64), ("rank", _i64), ("topk", _i64),
        ("local_window", _i64),
    ]
