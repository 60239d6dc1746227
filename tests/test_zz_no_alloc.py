"""GPU: the allocation-free verify entry point (std_verify_attn_noalloc).

It serves callers that may not allocate device memory -- a serving process
that keeps the whole GPU in its own pool, an FFI caller without a device
allocator, a loop that cannot afford an allocation's device synchronisation.
The test calls it through the C ABI twice in a row and checks each result
against the workspace entry point (std_verify_attn) on the same inputs, with
the attention tolerance the other tests use.  This file is collected last.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ATOL_MAX, ATOL_MEAN = 2e-2, 2e-3
SCRATCH_LIMIT = 32 << 20


def test_verify_noalloc_matches_workspace_entry_point():
    from std_b200 import _lib, ops

    lib = _lib.load()
    g = torch.Generator(device="cuda").manual_seed(21)
    B, nq, cap = 2, 10, 4096
    q = torch.randn(B, nq, 28, 128, generator=g, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, 4, cap, 128, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, 4, cap, 128, generator=g, device="cuda").to(torch.bfloat16)
    lens = torch.tensor([3000, 1500], dtype=torch.int32, device="cuda")
    ref_lse = torch.empty(B, nq, 28, dtype=torch.float32, device="cuda")
    ref = ops.verify_attention(q, k, v, lens, nq, lse=ref_lse)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        out = torch.full_like(q, float("nan"))
        lse = torch.empty(B, nq, 28, dtype=torch.float32, device="cuda")
        rc = lib.std_verify_attn_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens.data_ptr(), nq, nq, 1, B, 28,
                                         4, 128, cap, out.data_ptr(), lse.data_ptr(), stream)
        assert rc == 0
        torch.cuda.synchronize()
        err = (out.float() - ref.float()).abs()
        assert err.max().item() <= ATOL_MAX and err.mean().item() <= ATOL_MEAN
        assert (lse - ref_lse).abs().max().item() < 1e-3
    assert ops.device_error() == 0


def test_verify_noalloc_rejects_oversized_shapes():
    from std_b200 import _lib

    lib = _lib.load()
    B, Hkv, cap = 148, 4, 2048  # 592 CTAs of split partials: more than the fixed scratch holds
    assert lib.std_verify_attn_workspace_bytes(B, Hkv, cap) > SCRATCH_LIMIT
    rc = lib.std_verify_attn_noalloc(None, None, None, None, 0, 1, 1, B, 28, Hkv, 128, cap, None, None, None)
    assert rc == 2
