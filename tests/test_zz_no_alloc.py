"""Allocation-free paged decode attention, called through its exported C symbol.

The entry point serves callers that cannot allocate device memory (for example a host framework
that owns all device memory through its own pool, or a serving loop that must not pay for the
device-wide synchronisation of cudaMalloc / cudaFree); it keeps its split-KV partials in a fixed
device array inside the library.  This test
calls it twice in a row with different inputs and checks each result against the regular entry
point (which uses a caller-allocated workspace) and against the fp32 PyTorch oracle, within the
decode-attention test tolerance; it also covers a sequence exactly max_context long where
max_context is not a multiple of the 128-token split, and a second GPU in the same process.
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


def _call(fn, q, kc, vc, bt, lens, max_ctx):
    out = torch.empty_like(q)
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(), q.shape[0], q.shape[1],
            kc.shape[1], kc.shape[2], bt.shape[1], max_ctx, 1.0 / math.sqrt(128), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, out


def _err(a, b):
    return (a.float() - b.float()).abs().max().item()


def test_noalloc_matches_workspace_entry_point_twice():
    from axrl_b200.ops.paged import DecodeWorkspace, decode_attention_ref, paged_decode_attention

    fn = _lib()
    max_ctx = 24 * 64
    for seed in (0, 1):
        q, kc, vc, bt, lens = _case(seed)
        B, Hq = q.shape[0], q.shape[1]
        ref = paged_decode_attention(q, kc, vc, bt, lens, DecodeWorkspace(B, Hq, max_ctx, "cuda"))
        oracle = decode_attention_ref(q, kc, vc, bt, lens, 1.0 / math.sqrt(128))
        rc, out = _call(fn, q, kc, vc, bt, lens, max_ctx)
        assert rc == 0
        assert _err(out, ref) <= 2e-2, f"call {seed}: max err vs workspace entry {_err(out, ref)}"
        assert _err(out, oracle) <= 2e-2, f"call {seed}: max err vs fp32 oracle {_err(out, oracle)}"


def test_noalloc_sequence_at_max_context_not_multiple_of_split():
    """max_context = 1000 (not a multiple of 128) with one sequence exactly that long."""
    from axrl_b200.ops.paged import decode_attention_ref

    fn = _lib()
    q, kc, vc, bt, lens = _case(3, max_pages=16)  # 16 pages x 64 = 1024 >= 1000
    lens.copy_(torch.tensor([1000, 999, 1, 128, 640, 1000], dtype=torch.int32, device="cuda"))
    rc, out = _call(fn, q, kc, vc, bt, lens, 1000)
    assert rc == 0
    oracle = decode_attention_ref(q, kc, vc, bt, lens, 1.0 / math.sqrt(128))
    assert _err(out, oracle) <= 2e-2


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs in one process")
def test_noalloc_on_two_devices():
    from axrl_b200.ops.paged import decode_attention_ref

    fn = _lib()
    for dev in (0, 1, 0):
        with torch.cuda.device(dev):
            q, kc, vc, bt, lens = _case(4 + dev)
            rc, out = _call(fn, q, kc, vc, bt, lens, 24 * 64)
            assert rc == 0, f"device {dev}: rc {rc}"
            oracle = decode_attention_ref(q, kc, vc, bt, lens, 1.0 / math.sqrt(128))
            assert _err(out, oracle) <= 2e-2


def test_noalloc_rejects_oversized_call():
    fn = _lib()
    q, kc, vc, bt, lens = _case(2)
    out = torch.empty_like(q)
    rc = fn(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(), 6, 32, 8, 64, 1000, 64000,
            0.088, torch.cuda.current_stream().cuda_stream)
    assert rc == 1
