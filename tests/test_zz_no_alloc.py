"""GPU: the allocation-free verify entry point (std_verify_attn_noalloc).

It serves callers that may not allocate device memory -- a serving process
that keeps the whole GPU in its own pool, an FFI caller without a device
allocator, a loop that cannot afford an allocation's device synchronisation.
It runs the same kernels as the workspace entry point (std_verify_attn) with
the same split boundaries, so its output must equal that entry point's bit for
bit.  The test calls it through the C ABI on one shape, then on a larger shape
that writes split partials into more of the shared scratch array, then on the
first shape again: a merge that read a partial left over from the larger call
would show up as a mismatch on the third call.  This file is collected last.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu
SCRATCH_LIMIT = 32 << 20


def _inputs(seed, B, cap, lens):
    g = torch.Generator(device="cuda").manual_seed(seed)
    nq = 10
    q = torch.randn(B, nq, 28, 128, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, 4, cap, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, 4, cap, 128, generator=g, device="cuda").to(torch.bfloat16)
    return q, k, v, torch.tensor(lens, dtype=torch.int32, device="cuda")


def _noalloc(lib, q, k, v, lens):
    B, nq = q.shape[:2]
    cap = k.shape[2]
    out = torch.full_like(q, float("nan"))
    lse = torch.full((B, nq, 28), float("nan"), dtype=torch.float32, device="cuda")
    rc = lib.std_verify_attn_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), nq, nq, 1, B, 28, 4,
                                     128, cap, out.data_ptr(), lse.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    return out, lse


def _workspace(q, k, v, lens):
    from std_b200 import ops

    B, nq = q.shape[:2]
    lse = torch.empty(B, nq, 28, dtype=torch.float32, device="cuda")
    out = ops.verify_attention(q, k, v, lens, nq, lse=lse)
    torch.cuda.synchronize()
    return out, lse


def test_verify_noalloc_matches_workspace_entry_point():
    from std_b200 import _lib, ops

    lib = _lib.load()
    small = _inputs(21, 2, 4096, [3000, 1500])
    large = _inputs(22, 6, 8192, [8182, 8100, 7000, 8182, 4000, 8150])  # more splits and slots than `small`
    ref_small = _workspace(*small)
    ref_large = _workspace(*large)
    for inputs, ref in ((small, ref_small), (large, ref_large), (small, ref_small)):
        out, lse = _noalloc(lib, *inputs)
        assert torch.equal(out, ref[0])
        assert torch.equal(lse, ref[1])
    assert ops.device_error() == 0


def test_verify_noalloc_rejects_oversized_shapes():
    from std_b200 import _lib

    lib = _lib.load()
    B, Hkv, cap = 148, 4, 2048  # 592 CTAs of split partials: more than the fixed scratch holds
    assert lib.std_verify_attn_workspace_bytes(B, Hkv, cap) > SCRATCH_LIMIT
    rc = lib.std_verify_attn_noalloc(None, None, None, None, 0, 1, 1, B, 28, Hkv, 128, cap, None, None, None)
    assert rc == 2
    # a bad argument is reported as such (status 1) even when the shape is also too large
    rc = lib.std_verify_attn_noalloc(None, None, None, None, 0, 1, 1, B, 28, Hkv, 64, cap, None, None, None)
    assert rc == 1
