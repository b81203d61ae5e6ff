"""The allocation-free INT8 attention entry point matches the workspace one.

``sb_int8_sdpa_decode_static`` is for callers that cannot allocate device
memory (they only receive input and output buffers, or allocate nothing after
start-up): its split-K scratch is an array inside the library. This test calls
it through the C ABI twice in a row, on different shapes, and compares each
result with ``sb_int8_sdpa_decode`` given a caller workspace. The second call
also checks that whatever the first call left in the shared array does not
leak into the next result. This file is collected last so a failure here never
hides the other tests; it passes alone in a fresh process and after them.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from _util import assert_close  # noqa: E402

pytestmark = pytest.mark.gpu


def _inputs(seed, batch, heads, kv_heads, length, capacity):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(batch, heads, 1, 128, generator=g, device="cuda").bfloat16()
    k = torch.randint(-127, 128, (batch, kv_heads, capacity, 128), generator=g, device="cuda", dtype=torch.int8)
    v = torch.randint(-127, 128, (batch, kv_heads, capacity, 128), generator=g, device="cuda", dtype=torch.int8)
    ks = (torch.rand(batch, kv_heads, capacity, generator=g, device="cuda") * 0.02 + 0.005).half()
    vs = (torch.rand(batch, kv_heads, capacity, generator=g, device="cuda") * 0.02 + 0.005).half()
    return q, k, ks, v, vs


def test_static_scratch_sdpa_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import check, lib

    L = lib()
    stream = torch.cuda.current_stream().cuda_stream
    scale = 128 ** -0.5
    # two calls in a row: both use several token splits (the scratch is exercised)
    for seed, (batch, heads, kv_heads, length, capacity) in enumerate([(1, 32, 8, 4096, 4096),
                                                                       (2, 32, 8, 1000, 1024)]):
        q, k, ks, v, vs = _inputs(seed, batch, heads, kv_heads, length, capacity)
        assert L.sb_int8_sdpa_workspace_size(batch, heads, kv_heads, length, 128) > (128 << 10)  # splits > 1
        ws_bytes = L.sb_int8_sdpa_workspace_size(batch, heads, kv_heads, length, 128)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
        ref_out = torch.empty_like(q)
        check(L.sb_int8_sdpa_decode(q.data_ptr(), k.data_ptr(), ks.data_ptr(), v.data_ptr(), vs.data_ptr(),
                                    ref_out.data_ptr(), batch, heads, kv_heads, length, capacity, 128, scale,
                                    ws.data_ptr(), ws_bytes, stream), "sb_int8_sdpa_decode")
        out = torch.full_like(q, float("nan"))
        check(L.sb_int8_sdpa_decode_static(q.data_ptr(), k.data_ptr(), ks.data_ptr(), v.data_ptr(), vs.data_ptr(),
                                           out.data_ptr(), batch, heads, kv_heads, length, capacity, 128, scale,
                                           stream), "sb_int8_sdpa_decode_static")
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert_close(out.float().cpu().numpy(), ref_out.float().cpu().numpy(), what="static-scratch sdpa")


def test_static_scratch_rejects_oversized_shapes():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import lib

    L = lib()
    # batch 256 x 8 KV heads needs more split-K scratch than the 4 MiB array holds
    assert L.sb_int8_sdpa_workspace_size(256, 32, 8, 32768, 128) > (4 << 20)
    status = L.sb_int8_sdpa_decode_static(None, None, None, None, None, None, 256, 32, 8, 32768, 32768, 128,
                                          0.088, torch.cuda.current_stream().cuda_stream)
    assert status == 1  # SB_EINVAL, nothing launched
    assert b"static scratch holds" in L.sb_last_error_message()
    np.testing.assert_equal(status, 1)
