"""Summation order fixed across tensor-parallel degrees, checked on one GPU.

Greedy tokens are bit-identical at TP 1/2/4/8 only if every output element is
rounded from the same fp32 operations whatever the degree. Each piece of the
decoder that a shard computes is compared bit for bit here with the unsharded
launch it must reproduce:

* row-split o/down projections (``sb_linear_ex`` ``k_chunks``): the fp32 partial
  of each of the 8 K chunks is the same whether the launch covers all 8
  chunks (TP 1), 4 or 2 of them (a TP 2 / TP 4 rank) or one chunk alone (a TP 8
  rank); the output is the chunks' balanced-tree sum, which is also the order
  in which the fused exchange adds the ranks' partials;
* column-split QKV, gate/up and lm_head (``plan_rows``): a shard's rows equal the
  same rows of the unsharded launch;
* attention (``plan_kv_heads``): one KV head's group equals that group in the
  launch over all KV heads.
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CHUNKS = 8


def _need_cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")


def _bits(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _round_bf16(a):
    from oracle import formats

    return formats.round_bf16(np.asarray(a, dtype=np.float32))


def _tree(parts):
    """Balanced binary tree in index order (fp32): the kernel's chunk/rank sum."""
    v = [np.asarray(p, dtype=np.float32) for p in parts]
    s = 1
    while s < len(v):
        for i in range(0, len(v) - s, 2 * s):
            v[i] = (v[i] + v[i + s]).astype(np.float32)
        s *= 2
    return v[0]


def _row_split_weights(fmt, n, k, gen):
    """Weights [n, k] of the o (int8 per channel) or down (affine 4-bit G64) form,
    and a function giving the K columns [c0, c1) as contiguous tensors."""
    from spark_b200 import quantize

    w = torch.randn(n, k, generator=gen, device="cuda") * 0.02
    if fmt == "i8pc":
        codes, scale = quantize.quantize_w8_per_channel(w)

        def cols(c0, c1):
            return dict(weight_format=2, weight=codes[:, c0:c1].contiguous(), scales=scale)
        return cols
    packed, scales, biases = quantize.quantize_affine_minmax(w, 64, 4)

    def cols(c0, c1, pad=False):
        s, b = scales[:, c0 // 64:c1 // 64], biases[:, c0 // 64:c1 // 64]
        out = dict(weight_format=0, group_size=64, weight=packed[:, c0 // 8:c1 // 8].contiguous())
        if pad:  # table rows padded to a multiple of 8 groups (the decoder's TMA-able copy)
            ld = -(-s.shape[1] // 8) * 8
            sp = torch.zeros(n, ld, dtype=s.dtype, device=s.device)
            bp = torch.zeros_like(sp)
            sp[:, :s.shape[1]] = s
            bp[:, :s.shape[1]] = b
            return dict(out, scales=sp, biases=bp, scales_ld=ld)
        return dict(out, scales=s.contiguous(), biases=b.contiguous())
    return cols


def _launch(x, n, k, w, *, epilogue, y, residual=None, k_chunks=0, plan_k_chunks=0, plan_rows=0, norm=None):
    """One sb_linear_ex launch (fp32 output when y is fp32)."""
    from spark_b200._lib import check, lib, sb_linear_ex_desc

    keep = []
    fields = {}
    for key, val in w.items():
        if torch.is_tensor(val):
            keep.append(val)
            fields[key] = val.data_ptr()
        else:
            fields[key] = val
    m = x.shape[0]
    d = sb_linear_ex_desc(x=x.data_ptr(), x_dtype=0, ldx=x.stride(0), M=m, N=n, K=k, epilogue=epilogue,
                          y=y.data_ptr(), residual=residual.data_ptr() if residual is not None else None,
                          norm_weight=norm.data_ptr() if norm is not None else None, norm_eps=1e-6,
                          k_chunks=k_chunks, plan_k_chunks=plan_k_chunks, plan_rows=plan_rows,
                          y_fp32=int(y.dtype == torch.float32), **fields)
    ws = torch.zeros(max(lib().sb_linear_ex_workspace_size(ctypes.byref(d)), 256), dtype=torch.uint8, device="cuda")
    d.workspace, d.workspace_bytes = ws.data_ptr(), ws.numel()
    check(lib().sb_linear_ex(ctypes.byref(d), torch.cuda.current_stream().cuda_stream), "linear_ex")
    torch.cuda.synchronize()
    del keep


@pytest.mark.parametrize("fmt,n,k", [("i8pc", 2560, 4096), ("aff4", 2560, 9728)])
@pytest.mark.parametrize("m", [1, 8])
def test_row_split_chunks_identical_at_every_degree(fmt, n, k, m):
    _need_cuda()
    gen = torch.Generator(device="cuda").manual_seed(7 + m + (fmt == "aff4"))
    cols = _row_split_weights(fmt, n, k, gen)
    x = torch.randn(m, k, generator=gen, device="cuda").bfloat16()
    res = torch.randn(m, n, generator=gen, device="cuda").bfloat16()
    kc = k // CHUNKS

    def rank_partial(c0, c, **pad):
        """fp32 partial of chunks [c0, c0 + c): a TP (8 / c) rank's launch."""
        y = torch.empty(m, n, device="cuda", dtype=torch.float32)
        xs = x[:, c0 * kc:(c0 + c) * kc].contiguous()
        _launch(xs, n, c * kc, cols(c0 * kc, (c0 + c) * kc, **pad), epilogue=0, y=y, k_chunks=c if c > 1 else 0,
                plan_k_chunks=CHUNKS)
        return y.cpu().numpy()

    chunk = [rank_partial(c0, 1) for c0 in range(CHUNKS)]  # TP 8 ranks
    if fmt == "aff4":  # the same ranks with TMA-able (padded) scale tables
        for c0 in (0, 3, 7):
            assert np.array_equal(rank_partial(c0, 1, pad=True).view(np.uint32), chunk[c0].view(np.uint32)), c0
            assert np.array_equal(rank_partial(c0 // 2 * 2, 2, pad=True).view(np.uint32),
                                  _tree(chunk[c0 // 2 * 2:c0 // 2 * 2 + 2]).view(np.uint32)), c0
    full = rank_partial(0, CHUNKS)                           # TP 1
    assert np.array_equal(full.view(np.uint32), _tree(chunk).view(np.uint32)), "TP1 = tree of the 8 chunk partials"
    for c in (4, 2):                                         # TP 2 and TP 4 ranks: their subtrees
        for c0 in range(0, CHUNKS, c):
            got = rank_partial(c0, c)
            assert np.array_equal(got.view(np.uint32), _tree(chunk[c0:c0 + c]).view(np.uint32)), (c, c0)
    # the residual epilogue rounds the tree sum as the fused exchange does
    y1 = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    _launch(x, n, k, cols(0, k), epilogue=1, y=y1, residual=res, k_chunks=CHUNKS, plan_k_chunks=CHUNKS)
    want = _round_bf16(res.float().cpu().numpy() + _round_bf16(full))
    assert np.array_equal(_bits(y1), _bits(torch.from_numpy(want).bfloat16())), "tree sum + residual"


def test_chunks_agree_with_unchunked_values():
    """Chunking changes only the fp32 summation order: the result stays within a
    few bf16 ulps of the unchunked launch (and of the per-op tolerance)."""
    _need_cuda()
    gen = torch.Generator(device="cuda").manual_seed(3)
    n, k, m = 2560, 9728, 1
    cols = _row_split_weights("aff4", n, k, gen)
    x = torch.randn(m, k, generator=gen, device="cuda").bfloat16()
    y0 = torch.empty(m, n, device="cuda", dtype=torch.float32)
    y1 = torch.empty_like(y0)
    _launch(x, n, k, cols(0, k), epilogue=0, y=y0)
    _launch(x, n, k, cols(0, k), epilogue=0, y=y1, k_chunks=CHUNKS)
    a, b = y0.cpu().numpy(), y1.cpu().numpy()
    assert np.all(np.abs(a - b) <= 1e-5 + 1e-4 * np.abs(a))


@pytest.mark.parametrize("kind", ["qkv", "gateup", "head"])
@pytest.mark.parametrize("world", [2, 8])
def test_column_split_shard_rows_identical(kind, world):
    _need_cuda()
    from spark_b200 import quantize

    gen = torch.Generator(device="cuda").manual_seed(40 + world)
    k = 2560
    m = 1
    x = torch.randn(m, k, generator=gen, device="cuda").bfloat16()
    norm = (1.0 + 0.1 * torch.randn(k, generator=gen, device="cuda")).bfloat16()
    if kind == "qkv":
        n = 6144
        codes, scale = quantize.quantize_w8_per_channel(torch.randn(n, k, generator=gen, device="cuda") * 0.02)

        def w_rows(r0, r1):
            return dict(weight_format=2, weight=codes[r0:r1].contiguous(), scales=scale[r0:r1].contiguous())
        epi, width = 0, n
    elif kind == "gateup":
        n = 9728
        g = quantize.quantize_affine_minmax(torch.randn(n, k, generator=gen, device="cuda") * 0.02, 64, 4)
        u = quantize.quantize_affine_minmax(torch.randn(n, k, generator=gen, device="cuda") * 0.02, 64, 4)

        def w_rows(r0, r1):
            return dict(weight_format=0, group_size=64, weight=g[0][r0:r1].contiguous(),
                        scales=g[1][r0:r1].contiguous(), biases=g[2][r0:r1].contiguous(),
                        weight2=u[0][r0:r1].contiguous(), scales2=u[1][r0:r1].contiguous(),
                        biases2=u[2][r0:r1].contiguous())
        epi, width = 2, n
    else:
        n = 151936
        head = (torch.randn(n, k, generator=gen, device="cuda") * 0.02).bfloat16()

        def w_rows(r0, r1):
            return dict(weight_format=3, weight=head[r0:r1].contiguous())
        epi, width = 0, n
    y_full = torch.empty(m, width, device="cuda", dtype=torch.bfloat16)
    _launch(x, n, k, w_rows(0, n), epilogue=epi, y=y_full, norm=norm)
    rows = n // world
    for r in (0, world - 1):
        ys = torch.empty(m, rows, device="cuda", dtype=torch.bfloat16)
        _launch(x, rows, k, w_rows(r * rows, (r + 1) * rows), epilogue=epi, y=ys, norm=norm, plan_rows=n)
        assert np.array_equal(_bits(ys), _bits(y_full[:, r * rows:(r + 1) * rows])), (kind, world, r)


@pytest.mark.parametrize("length", [1100, 4096])
def test_attention_shard_plans_like_all_heads(length):
    _need_cuda()
    from spark_b200._lib import check, lib

    b, hq, hkv, d, cap = 1, 32, 8, 128, ((length + 15) // 16) * 16
    gen = torch.Generator(device="cuda").manual_seed(length)
    q = torch.randn(b, hq, 1, d, generator=gen, device="cuda").bfloat16()
    kc = torch.randint(-127, 128, (b, hkv, cap, d), generator=gen, device="cuda", dtype=torch.int8)
    vc = torch.randint(-127, 128, (b, hkv, cap, d), generator=gen, device="cuda", dtype=torch.int8)
    ks = (torch.rand(b, hkv, cap, generator=gen, device="cuda") * 0.02 + 0.001).half()
    vs = (torch.rand(b, hkv, cap, generator=gen, device="cuda") * 0.02 + 0.001).half()
    lengths = torch.full((b,), length, dtype=torch.int32, device="cuda")
    nbytes = lib().sb_int8_sdpa_workspace_size(b, hq, hkv, cap, d)
    stream = torch.cuda.current_stream().cuda_stream

    def run(qq, kk, kss, vv, vss, heads, kv_heads, plan):
        out = torch.empty(b, heads, 1, d, device="cuda", dtype=torch.bfloat16)
        ws = torch.zeros(nbytes + 256, dtype=torch.uint8, device="cuda")
        check(lib().sb_int8_sdpa_decode_dev(qq.data_ptr(), kk.data_ptr(), kss.data_ptr(), vv.data_ptr(),
                                            vss.data_ptr(), out.data_ptr(), b, heads, kv_heads, lengths.data_ptr(), 0,
                                            cap, cap, d, 1.0 / np.sqrt(d), 0, plan, ws.data_ptr(), ws.numel(),
                                            stream), "sdpa")
        torch.cuda.synchronize()
        return out

    full = run(q, kc, ks, vc, vs, hq, hkv, 0)
    g = hq // hkv
    for world in (2, 8):
        hk = hkv // world
        for r in (0, world - 1):
            sl = slice(r * hk, (r + 1) * hk)
            qs = q[:, r * hk * g:(r + 1) * hk * g].contiguous()
            got = run(qs, kc[:, sl].contiguous(), ks[:, sl].contiguous(), vc[:, sl].contiguous(),
                      vs[:, sl].contiguous(), hk * g, hk, hkv)
            assert np.array_equal(_bits(got), _bits(full[:, r * hk * g:(r + 1) * hk * g])), (world, r)
