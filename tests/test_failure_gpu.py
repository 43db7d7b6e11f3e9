"""Failure detection on one GPU without a fault: a collective kernel whose peer never arrives.

The "peer" of each kernel below is a second buffer on the same GPU whose flags nothing writes, so every
bounded wait runs out after a 20 ms limit.  The kernels must then record the peer-timeout bit in the
status word the host reads (`_ext.check_status` raises `DeviceStepError`), return without hanging, and
leave the context usable: an ordinary kernel launched next gives the right result.  No kernel here
traps, faults or spins without a limit."""

import pytest
import torch

pytestmark = pytest.mark.gpu

PEER_TIMEOUT = 2


def _fresh_status():
    from vllm_cmp170hx_b200 import _ext

    w = _ext.status_word(torch.device("cuda", torch.cuda.current_device()))
    w.zero_()
    return w


def _ordinary_kernel_still_works():
    from vllm_cmp170hx_b200 import _ext, ops

    x = torch.randn(64, 256, device="cuda").bfloat16()
    w = torch.randn(512, 256, device="cuda").bfloat16()
    y = ops.gemm(x, w)
    torch.cuda.synchronize()
    ref = x.float() @ w.float().t()
    assert ((y.float() - ref).norm() / ref.norm()).item() < 1e-2
    _ext.check_status(x.device)  # nothing new recorded


def test_one_shot_all_reduce_peer_never_arrives():
    from vllm_cmp170hx_b200 import _ext

    st = _fresh_status()
    flag_bytes, half = 64 * 1024, 1 << 20
    bufs = [torch.zeros(flag_bytes + 2 * half, dtype=torch.uint8, device="cuda") for _ in range(2)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    epochs = torch.zeros(8, dtype=torch.int32, device="cuda")
    x = torch.randn(4096, device="cuda").bfloat16()
    out = torch.empty_like(x)
    _ext.ops().symm_all_reduce(x, out, peers, 0, 2, flag_bytes, half, epochs, st, 0.02)
    torch.cuda.synchronize()
    assert int(st.item()) & PEER_TIMEOUT
    with pytest.raises(_ext.DeviceStepError, match="peer flag wait timed out"):
        _ext.check_status(x.device)
    _ordinary_kernel_still_works()


def _lonely_sync():
    """Sequence-parallel buffers of a two-rank group whose second rank is a local stand-in."""
    from vllm_cmp170hx_b200.parallel.sp import FLAG_BYTES

    size = FLAG_BYTES + (8 << 20)
    bufs = [torch.zeros(size, dtype=torch.uint8, device="cuda") for _ in range(2)]
    peers = torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")
    state = torch.zeros(16, dtype=torch.int32, device="cuda")
    return bufs, peers, state


@pytest.mark.parametrize("channel", [0, 1, 2, 3])
def test_sp_wait_peer_never_arrives(channel):
    from vllm_cmp170hx_b200 import _ext

    st = _fresh_status()
    bufs, peers, state = _lonely_sync()
    _ext.ops().sp_wait(peers, 0, state, st, 0.02, channel)
    torch.cuda.synchronize()
    assert int(st.item()) & PEER_TIMEOUT
    # the call still counted as received: the next call waits for the next number
    assert int(state.view(4, 4)[channel, 2].item()) == 1
    st.zero_()
    _ordinary_kernel_still_works()


def test_all_gather_gemm_peer_never_arrives():
    """The GEMM whose producer waits for the all-gather gives up after the limit, finishes its tiles
    (with whatever rows are there) and reports the timeout."""
    from vllm_cmp170hx_b200 import _ext
    from vllm_cmp170hx_b200.parallel.sp import FLAG_BYTES

    st = _fresh_status()
    bufs, peers, state = _lonely_sync()
    T, K, N = 16, 512, 1024
    x = bufs[0][FLAG_BYTES:FLAG_BYTES + T * K * 2].view(torch.bfloat16).view(T, K)
    w = torch.randn(N, K, device="cuda").bfloat16()
    out = torch.empty(T, N, dtype=torch.bfloat16, device="cuda")
    _ext.ops().gemm_sp(x, w, out, st, 0, peers, 0, state, 0.02, 2, 0, 0)
    torch.cuda.synchronize()
    assert int(st.item()) & PEER_TIMEOUT
    st.zero_()
    _ordinary_kernel_still_works()
