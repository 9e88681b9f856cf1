"""CPU: the C-ABI library builds, loads, exports every declared entry point,
and rejects bad arguments with error codes before touching a device."""

import ctypes as C
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "mrsa.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:const char\*|int|size_t)\s+(mrsa_\w+)\(", text, re.M)))


def test_header_lists_entry_points():
    names = _declared()
    assert "mrsa_route_layer_forward" in names and "mrsa_selected_attention" in names
    assert len(names) >= 14


def test_library_exports_every_declared_symbol(mrsa):
    lib_path = mrsa._lib.LIB_PATH
    assert os.path.exists(lib_path), "run __graft_entry__.build() first"
    out = subprocess.run(["nm", "-D", "--defined-only", lib_path], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(mrsa_\w+)\b", out))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    assert set(mrsa._lib.EXPORTED) == set(_declared())


def test_strerror_and_version(mrsa):
    lib = mrsa._lib.load()
    assert lib.mrsa_abi_version() == 3
    assert lib.mrsa_strerror(0) == b"ok"
    assert b"NULL" in lib.mrsa_strerror(-1)
    assert lib.mrsa_strerror(-99) == b"unknown error"


def test_bad_arguments_return_codes_without_device(mrsa):
    lib = mrsa._lib.load()
    dummy = C.c_void_p(4096)
    # NULL inputs
    assert lib.mrsa_rope(None, None, 28, None, None, 0, None, None, 1.0, None, None, 0, 1, 64, 128, None) == -1
    # unsupported head_dim
    assert lib.mrsa_rope(dummy, dummy, 28, None, None, 0, dummy, dummy, 1.0, None, None, 0, 1, 64, 64, None) == -2
    # misaligned pointer
    assert lib.mrsa_rope(C.c_void_p(4098), dummy, 28, None, None, 0, dummy, dummy, 1.0, None, None, 0,
                         1, 64, 128, None) == -3
    # topk > 32 and too many chunks are shape errors
    args = [dummy, dummy, 1, dummy, None, None, None, 256, 0, dummy, dummy, 0, None, None, 0, 1.0, 1.0,
            0.0, 1, 64, 4, 4, 7, 128]
    assert lib.mrsa_route_topk(*args, 33, dummy, 1 << 30, None) == -2
    args2 = list(args)
    args2[20] = 4096
    assert lib.mrsa_route_topk(*args2, 32, dummy, 1 << 30, None) == -2
    # bad temperature
    args3 = list(args)
    args3[15] = 0.0
    assert lib.mrsa_route_topk(*args3, 32, dummy, 1 << 30, None) == -5
    # the keys workspace: B*Lq*Hkv*C fp32, refused when missing or short
    # keys fp32 [B,Lq,Hkv,C] (256-byte rounded) + raw scores [B,Lq,Hq,C] in the scores dtype
    n = lib.mrsa_route_topk_workspace_size(1, 64, 4, 4, 7, 0)
    assert n == 64 * 4 * 4 * 4 + 64 * 28 * 4 * 2
    assert lib.mrsa_route_topk_workspace_size(1, 64, 4, 4, 7, 1) == 64 * 4 * 4 * 4 + 64 * 28 * 4 * 4
    assert lib.mrsa_route_topk_workspace_size(0, 64, 4, 4, 7, 0) == 0
    assert lib.mrsa_route_topk(*args, 32, None, 0, None) == -6
    assert lib.mrsa_route_topk(*args, 32, dummy, n - 1, None) == -6
    # selected attention: chunk must be 64, kv_len a multiple of it
    assert lib.mrsa_selected_attention(dummy, dummy, dummy, None, dummy, dummy, None, None, dummy, 0.1, 1,
                                       1, 64, 100, 4, 7, 128, 32, 64, None) == -2
    # local/weight must come together
    assert lib.mrsa_selected_attention(dummy, dummy, dummy, None, dummy, dummy, dummy, None, dummy, 0.1, 1,
                                       1, 64, 128, 4, 7, 128, 32, 64, None) == -1
    # tile-gather probe: missing status pointer, more than 8 owners, kv_len not whole chunks
    assert lib.mrsa_probe_tile_gather(dummy, dummy, dummy, 4096, 4, 64, 4, 10, None, None) == -1
    assert lib.mrsa_probe_tile_gather(dummy, dummy, dummy, 4096, 4, 64, 9, 10, dummy, None) == -2
    assert lib.mrsa_probe_tile_gather(dummy, dummy, dummy, 4000, 4, 64, 4, 10, dummy, None) == -2
    # route layer: workspace checks
    a = mrsa._lib.RouteLayerArgs()
    assert lib.mrsa_route_layer_workspace_size(C.byref(a)) == 0
    assert lib.mrsa_route_layer_forward(C.byref(a), None, 0, None) == -1


@pytest.mark.parametrize("l", [16384, 512])
def test_route_layer_workspace_size_formula(mrsa, l):
    lib = mrsa._lib.load()
    a = mrsa._lib.RouteLayerArgs()
    a.batch, a.seq_len, a.q_heads, a.kv_heads, a.head_dim = 1, l, 28, 4, 128
    a.hidden_size, a.rank, a.topk, a.local_window = 3584, 64, 32, 256
    n = lib.mrsa_route_layer_workspace_size(C.byref(a))
    hq, hkv, d, k, c = 28, 4, 128, 32, l // 64
    # q, route_q, local_out; k and its fp16 V; landmarks, prior, entropy, validity;
    # local LSE, indices, scores + remote weights, local weight; routing keys + raw scores
    expect = (3 * l * hq * d * 2 + 2 * l * hkv * d * 2 + c * hq * d * 2 + 2 * c * hq * 4 + c
              + l * hq * 4 + l * hkv * k * 4 + 2 * l * hq * k * 2 + l * hq * 2
              + l * hkv * c * 4 + l * hq * c * 2)
    assert expect <= n <= expect + 15 * 256


def test_yarn_host_table_matches_transformers(mrsa):
    import torch

    from conftest import load_golden

    g = load_golden("yarn.pt")
    lib = mrsa._lib.load()
    buf = (C.c_float * 64)()
    af = C.c_float()
    assert lib.mrsa_yarn_inv_freq(128, 1.0e6, 8.0, 2048, 32.0, 1.0, 1, buf, C.byref(af)) == 0
    got = torch.tensor(list(buf), dtype=torch.float32)
    torch.testing.assert_close(got, g["inv_freq"], rtol=2e-7, atol=0)
    assert af.value == pytest.approx(g["attention_factor"], rel=1e-7)
    inv, af2 = mrsa.yarn_inv_freq()
    assert torch.equal(inv, g["inv_freq"]) and af2 == g["attention_factor"]


def test_ops_raise_without_cuda_tensors(mrsa):
    import torch

    q = torch.zeros(1, 64, 28, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 64, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        mrsa.bidir_local_attention(q, k, k, torch.ones(1, 64, dtype=torch.bool), 256, 64)
    with pytest.raises(ValueError, match="CUDA"):
        mrsa.chunk_attn_pool_gqa(torch.zeros(1, 1, 4, 7, 128, dtype=torch.bfloat16),
                                 torch.zeros(1, 1, 64, 4, 128, dtype=torch.bfloat16),
                                 torch.ones(1, 1, 64, dtype=torch.bool))


def test_token_ops_and_flex_reject_bad_arguments(mrsa):
    lib = mrsa._lib.load()
    d = C.c_void_p(4096)
    # flex: q_len > kv_len is a shape error, chunk <= 0 and sm_scale <= 0 argument errors
    assert lib.mrsa_flex_attention(d, d, d, d, None, 64, 64, 1, 1, 0, 0.1, 1, 65, 64, 8, 2, 128, None) == -2
    assert lib.mrsa_flex_attention(d, d, d, d, None, 64, 0, 1, 1, 0, 0.1, 1, 64, 64, 8, 2, 128, None) == -5
    assert lib.mrsa_flex_attention(d, d, d, d, None, 64, 64, 1, 1, 0, 0.0, 1, 64, 64, 8, 2, 128, None) == -5
    assert lib.mrsa_flex_attention(d, d, d, d, None, 64, 64, 1, 1, -1, 0.1, 1, 64, 64, 8, 2, 128, None) == -5
    assert lib.mrsa_flex_attention(None, d, d, d, None, 64, 64, 1, 1, 0, 0.1, 1, 64, 64, 8, 2, 128, None) == -1
    # token scores: chunk < 16, kv_len not a multiple of chunk, head_dim != 128, groups > 16
    ts = [d, d, d, None, d, 0.1, 1, 4]
    assert lib.mrsa_candidate_token_scores(*ts, 256, 28, 4, 128, 2, 8, None) == -2
    assert lib.mrsa_candidate_token_scores(*ts, 250, 28, 4, 128, 2, 64, None) == -2
    assert lib.mrsa_candidate_token_scores(*ts, 256, 28, 4, 64, 2, 64, None) == -2
    assert lib.mrsa_candidate_token_scores(*ts, 256, 34, 2, 128, 2, 64, None) == -2
    assert lib.mrsa_candidate_token_scores(C.c_void_p(4100), d, d, None, d, 0.1, 1, 4, 256, 28, 4, 128, 2, 64,
                                           None) == -3
    # selected-token attention: NULL valid, groups > 16, shared memory beyond 227 KB
    assert lib.mrsa_selected_token_attention(d, d, d, d, None, d, 0.1, 1, 4, 256, 28, 4, 128, 8, None) == -1
    assert lib.mrsa_selected_token_attention(d, d, d, d, d, d, 0.1, 1, 4, 256, 34, 2, 128, 8, None) == -2
    assert lib.mrsa_selected_token_attention(d, d, d, d, d, d, 0.1, 1, 4, 256, 28, 4, 128, 20000, None) == -2
    assert lib.mrsa_selected_token_attention_smem(7, 2560) == 7 * 2560 * 4 + 2560 * 4 + 4 * 7 * 512
    assert lib.mrsa_selected_token_attention_smem(7, 101) == 7 * 104 * 4 + 104 * 4 + 4 * 7 * 512
    assert lib.mrsa_selected_token_attention_smem(17, 64) == 0


def test_local_attention_positions_needs_positions(mrsa):
    lib = mrsa._lib.load()
    d = C.c_void_p(4096)
    assert lib.mrsa_local_attention_positions(d, d, d, None, None, d, None, 256, 1, 64, 0.1, 1, 4, 256, 28, 4,
                                              128, None) == -1
    assert lib.mrsa_local_attention_positions(d, d, d, None, d, d, None, 256, 1, 64, 0.1, 1, 4, 256, 28, 4,
                                              64, None) == -2
