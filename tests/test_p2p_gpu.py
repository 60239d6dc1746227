"""The peer-exchange primitives of the sequence-sharded verify on one GPU:
std_p2p_post / std_p2p_wait (epoch flags, bounded waits) and
std_merge_partials_f32_list against std_merge_partials_f32.  Every wait here
follows its post in stream order on the same GPU, so no kernel spins on work
that has not been launched; the timeout case waits on a flag nothing sets and
must end with STD_DEVERR_WAIT_TIMEOUT after about a second, leaving the
context usable.  The cross-GPU path is tests/test_seq_shard_gpu.py."""
import ctypes
import time

import pytest
import torch

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT = 1


def _ptrs(*tensors):
    return (ctypes.c_ulonglong * len(tensors))(*[t.data_ptr() for t in tensors])


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_post_copies_then_publishes_and_wait_advances():
    from std_b200 import _lib, ops

    dev = torch.device("cuda", 0)
    ops.device_error()
    n = 2240 * 128  # one verify block's queries at B=8, nq=10
    flags = torch.zeros(4, dtype=torch.int32, device=dev)
    ctr = torch.zeros(4, dtype=torch.int32, device=dev)  # [post counter, wait counter]
    dst = torch.zeros(n, dtype=torch.bfloat16, device=dev)
    for epoch in (1, 2, 3):
        src = torch.randn(n, device=dev).to(torch.bfloat16)
        three = _ptrs(flags[0:1], flags[1:2], flags[2:3])
        _lib.call("std_p2p_post", src.data_ptr(), dst.data_ptr(), n * 2, three, 3, ctr[0:1].data_ptr(), _stream())
        _lib.call("std_p2p_wait", flags.data_ptr(), 3, ctr[1:2].data_ptr(), _stream())
        torch.cuda.synchronize()
        assert torch.equal(dst.view(torch.int16), src.view(torch.int16))
        assert flags[:3].tolist() == [epoch] * 3 and flags[3].item() == 0
        assert ctr[:2].tolist() == [epoch, epoch]
    # a flag-only post (a server's "partial ready")
    _lib.call("std_p2p_post", None, None, 0, _ptrs(flags[3:4]), 1, ctr[2:3].data_ptr(), _stream())
    torch.cuda.synchronize()
    assert flags[3].item() == 1 and ctr[2].item() == 1
    assert ops.device_error() == 0


def test_post_rejects_bad_arguments():
    from std_b200 import _lib

    dev = torch.device("cuda", 0)
    buf = torch.zeros(64, dtype=torch.int32, device=dev)
    flag = _ptrs(buf[0:1])
    s = _stream()
    with pytest.raises(RuntimeError):  # size not a multiple of 16
        _lib.call("std_p2p_post", buf.data_ptr(), buf[32:].data_ptr(), 24, flag, 1, buf[63:].data_ptr(), s)
    with pytest.raises(RuntimeError):  # misaligned source
        _lib.call("std_p2p_post", buf[1:].data_ptr(), buf[32:].data_ptr(), 16, flag, 1, buf[63:].data_ptr(), s)
    with pytest.raises(RuntimeError):  # more than 8 flags
        _lib.call("std_p2p_post", None, None, 0, _ptrs(*[buf[0:1]] * 9), 9, buf[63:].data_ptr(), s)
    with pytest.raises(RuntimeError):  # no flags to wait for
        _lib.call("std_p2p_wait", buf.data_ptr(), 0, buf[63:].data_ptr(), s)


def test_wait_on_unset_flag_times_out_and_context_survives():
    from std_b200 import _lib, ops

    dev = torch.device("cuda", 0)
    ops.device_error()
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    ctr = torch.zeros(2, dtype=torch.int32, device=dev)
    torch.cuda.synchronize()
    t0 = time.time()
    _lib.call("std_p2p_wait", flags.data_ptr(), 1, ctr.data_ptr(), _stream())
    torch.cuda.synchronize()
    waited = time.time() - t0
    assert 0.5 < waited < 30.0
    assert ops.device_error() == WAIT_TIMEOUT
    assert ctr[0].item() == 1  # the epoch advances anyway, so later steps stay in step
    # the context is still usable
    x = torch.arange(16, device=dev, dtype=torch.float32)
    assert float((x * 2).sum().item()) == 240.0
    _lib.call("std_p2p_post", None, None, 0, _ptrs(flags[1:2]), 1, ctr[1:2].data_ptr(), _stream())
    torch.cuda.synchronize()
    assert flags[1].item() == 1 and ops.device_error() == 0


@pytest.mark.parametrize("n_parts,rows", [(2, 280), (3, 2240), (8, 70)])
def test_merge_list_equals_packed_merge(n_parts, rows):
    from std_b200 import _lib, ops

    dev = torch.device("cuda", 0)
    D = 128
    g = torch.Generator(device=dev).manual_seed(7 + n_parts)
    stride = rows * (D + 1)
    packed = torch.randn(n_parts, stride, device=dev, generator=g)
    lse = packed[:, rows * D:]
    lse.mul_(3.0)
    lse[0, ::5] = float("-inf")                 # a part that sees no key of some rows
    lse[:, ::17] = float("-inf")                # rows no part sees
    parts = [packed[i].clone() for i in range(n_parts)]  # separate allocations, as on separate GPUs
    out_a = torch.empty(rows, D, dtype=torch.bfloat16, device=dev)
    out_b = torch.empty_like(out_a)
    lse_a = torch.empty(rows, device=dev)
    lse_b = torch.empty(rows, device=dev)
    ops.merge_partials_f32(packed, rows, D, out_a, lse_a)
    _lib.call("std_merge_partials_f32_list", _ptrs(*parts), n_parts, rows, D, out_b.data_ptr(), lse_b.data_ptr(),
              _stream())
    torch.cuda.synchronize()
    assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16))
    assert torch.equal(lse_a.view(torch.int32), lse_b.view(torch.int32))


def test_exported_allocation_round_trip():
    from std_b200 import _lib

    torch.cuda.set_device(0)
    hb = int(_lib.query("std_ipc_handle_bytes"))
    assert hb == 64
    ptr = ctypes.c_void_p(0)
    _lib.call("std_device_alloc", 4096, ctypes.byref(ptr))
    try:
        buf = ctypes.create_string_buffer(hb)
        _lib.call("std_ipc_handle", ptr.value, buf)
        assert any(buf.raw)
    finally:
        _lib.call("std_device_free", ptr.value)
