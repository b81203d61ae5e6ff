"""A bounded device-side wait that runs out reports a timeout and leaves the
CUDA context usable (failure detection without a GPU fault).

The fused tensor-parallel all-reduce of the o/down projection epilogue waits,
per output element, for the other ranks' partial sums to appear in this rank's
exchange buffer. Here a single process launches it as rank 0 of 2 and no rank
1 ever writes: every wait gives up after its bound (about a second), the kernel
sets the timeout bit in the workspace status word and returns. The test checks
the status word, that this rank's own partials still reached the "peer"
buffer, and that the same projection then runs correctly without the
exchange.
"""

import ctypes
import time

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import formats  # noqa: E402

from _util import assert_close  # noqa: E402

pytestmark = pytest.mark.gpu

STATUS_WORD = 128 * 1024 // 4 - 1  # last word of the workspace counter region
STATUS_TIMEOUT = 1


def test_fused_allreduce_wait_gives_up_and_reports_timeout():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import check, lib, sb_linear_ex_desc

    L = lib()
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    n, k = 64, 256
    w = torch.randint(-127, 128, (n, k), generator=g, device=dev, dtype=torch.int8)
    s = (torch.rand(n, generator=g, device=dev) * 0.01 + 0.001).float()
    x = torch.randn(1, k, generator=g, device=dev).bfloat16()
    resid = torch.randn(1, n, generator=g, device=dev).bfloat16()
    y = torch.empty(1, n, device=dev, dtype=torch.bfloat16)
    xbytes = L.sb_tp_exchange_bytes(2, n)
    own = torch.zeros(xbytes, dtype=torch.uint8, device=dev)   # rank 1 would write here; nobody does
    peer = torch.zeros(xbytes, dtype=torch.uint8, device=dev)  # stands in for rank 1's buffer

    d = sb_linear_ex_desc(x=x.data_ptr(), x_dtype=0, M=1, N=n, K=k, weight_format=2, weight=w.data_ptr(),
                          scales=s.data_ptr(), epilogue=1, y=y.data_ptr(), residual=resid.data_ptr(),
                          weights_constant=1, ar_world=2, ar_rank=0, ar_channel=0)
    d.ar_buffers[0] = own.data_ptr()
    d.ar_buffers[1] = peer.data_ptr()
    ws_bytes = L.sb_linear_ex_workspace_size(ctypes.byref(d))
    ws = torch.zeros(max(ws_bytes, 128 * 1024), dtype=torch.uint8, device=dev)
    d.workspace = ws.data_ptr()
    d.workspace_bytes = ws.numel()
    stream = torch.cuda.current_stream().cuda_stream

    t0 = time.perf_counter()
    check(L.sb_linear_ex(ctypes.byref(d), stream), "linear with a missing peer")
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    status = int(ws.view(torch.int32)[STATUS_WORD].item())
    assert status & STATUS_TIMEOUT, status
    assert elapsed < 60.0, elapsed  # bounded: the waits gave up
    assert bool(peer.any())         # this rank still posted its partial sums

    # the context still works: the same projection without the exchange
    ws.zero_()
    d.ar_world = 0
    check(L.sb_linear_ex(ctypes.byref(d), stream), "linear")
    torch.cuda.synchronize()
    assert int(ws.view(torch.int32)[STATUS_WORD].item()) == 0
    acc = x.float().cpu().numpy().astype(np.float64) @ w.cpu().numpy().astype(np.float64).T
    part = formats.round_bf16((acc * s.cpu().numpy().astype(np.float64)).astype(np.float32))
    expected = resid.float().cpu().numpy() + part
    assert_close(y.float().cpu().numpy(), expected, what="linear after a timed-out exchange")


def test_tp_decoder_raises_when_a_peer_never_posts(monkeypatch):
    """A tensor-parallel decoder whose peer never posts its o/down partial sums
    raises instead of returning tokens, and within a few seconds: the first
    wait that runs out sets the status word and every later wait (also in
    later launches) is skipped. One process plays rank 0 of 2; the 'peer'
    exchange buffer is a local buffer that nobody writes."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import SBError, lib
    from spark_b200.decoder import DecoderConfig, SyntheticDecoder

    def local_exchange(self):
        nbytes = lib().sb_tp_exchange_bytes(self.world, self.cfg.hidden)
        self._fake_buffers = [torch.zeros(nbytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.ar_buffers = [b.data_ptr() for b in self._fake_buffers]
        self._own_buffer, self._mapped = None, []

    monkeypatch.setattr(SyntheticDecoder, "_setup_exchange", local_exchange)
    monkeypatch.setattr(SyntheticDecoder, "_allreduce", lambda self, t, op=None: None)
    dec = SyntheticDecoder(DecoderConfig.small(num_layers=4), batch=1, capacity=32, rank=0, world=2, group=None)
    dec.reset([1])
    t0 = time.perf_counter()
    with pytest.raises(SBError, match="gave up"):
        dec.decode(3)
    assert time.perf_counter() - t0 < 30.0
    dec.check_status()  # cleared by the raise: no second report
