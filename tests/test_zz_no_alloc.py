"""Allocation-free paged decode attention, called through its exported C symbol.

The entry point serves callers that cannot allocate device memory (for example a host framework
that owns all device memory through its own pool, or a serving loop that must not pay for the
device-wide synchronisation of cudaMalloc / cudaFree); it keeps its split-KV partials in a fixed
device array inside the library.  This test
calls it twice in a row with different inputs and checks each result against the regular entry
point (which uses a caller-allocated workspace) within the decode-attention test tolerance.
"""

import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from axrl_b200.ops import _ext

    _ext.ext()  # loads the extension (and libtorch) into the process first
    lib = ctypes.CDLL(_ext._so_path("_C"))
    fn = lib.axrl_paged_decode_attention_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_float, ctypes.c_void_p]
    return fn


def _case(seed, B=6, Hq=32, Hkv=8, P=64, pages=80, max_pages=24):
    g = torch.Generator(device="cuda").manual_seed(seed)
    kc = torch.randn(pages, Hkv, P, 128, device="cuda", generator=g).bfloat16()
    vc = torch.randn(pages, Hkv, P, 128, device="cuda", generator=g).bfloat16()
    lens = torch.tensor([1, 40, 64, 65, 700, 1500][:B], dtype=torch.int32, device="cuda")
    bt = torch.randint(0, pages, (B, max_pages), dtype=torch.int32, device="cuda", generator=g)
    q = torch.randn(B, Hq, 128, device="cuda", generator=g).bfloat16()
    return q, kc, vc, bt, lens


def test_noalloc_matches_workspace_entry_point_twice():
    from axrl_b200.ops.paged import DecodeWorkspace, paged_decode_attention

    fn = _lib()
    max_ctx = 24 * 64
    for seed in (0, 1):
        q, kc, vc, bt, lens = _case(seed)
        B, Hq = q.shape[0], q.shape[1]
        ref = paged_decode_attention(q, kc, vc, bt, lens, DecodeWorkspace(B, Hq, max_ctx, "cuda"))
        out = torch.empty_like(q)
        rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(), B, Hq, kc.shape[1],
                kc.shape[2], bt.shape[1], max_ctx, 1.0 / math.sqrt(128), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 2e-2, f"call {seed}: max err {err}"


def test_noalloc_rejects_oversized_call():
    fn = _lib()
    q, kc, vc, bt, lens = _case(2)
    out = torch.empty_like(q)
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(), 6, 32, 8, 64, 1000, 64000,
            0.088, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
