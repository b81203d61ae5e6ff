"""The QKV kernel's fused INT8 cache append equals the two-kernel path
(store K/V in bf16, then sb_kv_append_int8) bit for bit."""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bsz,hq,hkv,d,k,parts_hint", [(2, 8, 2, 128, 1024, "few"), (3, 4, 2, 64, 2560, "many"),
                                                       (1, 32, 8, 128, 2560, "decoder")])
def test_fused_cache_append_matches_kv_append(bsz, hq, hkv, d, k, parts_hint):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from spark_b200._lib import check, lib, sb_linear_ex_desc
    from spark_b200.quantize import quantize_w8_per_channel

    L = lib()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(bsz * 100 + d)
    n = (hq + 2 * hkv) * d
    wq, ws = quantize_w8_per_channel(torch.randn(n, k, generator=g, device=dev) * 0.02)
    x = torch.randn(bsz, k, generator=g, device=dev).bfloat16()
    norm = (1 + 0.1 * torch.randn(k, generator=g, device=dev)).bfloat16()
    capacity = 48
    positions = torch.tensor([5, 17, 47][:bsz], dtype=torch.int32, device=dev)
    work = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)

    def caches():
        kc = torch.full((bsz, hkv, capacity, d), 3, dtype=torch.int8, device=dev)
        ksc = torch.full((bsz, hkv, capacity), 2.0, dtype=torch.float16, device=dev)
        return kc, ksc, kc.clone(), ksc.clone()

    q_a = torch.empty(bsz, hq, 1, d, dtype=torch.bfloat16, device=dev)
    q_b = torch.empty_like(q_a)
    k_new = torch.empty(bsz, hkv, 1, d, dtype=torch.bfloat16, device=dev)
    v_new = torch.empty_like(k_new)

    def desc(q_out, fused):
        dsc = sb_linear_ex_desc(x=x.data_ptr(), x_dtype=0, M=bsz, N=n, K=k, weight_format=2, weight=wq.data_ptr(),
                                scales=ws.data_ptr(), norm_weight=norm.data_ptr(), norm_eps=1e-6, epilogue=3,
                                positions=positions.data_ptr(), num_heads=hq, num_kv_heads=hkv, head_dim=d,
                                seq_len=1, rope_base=1e6, q_out=q_out.data_ptr(), k_out=k_new.data_ptr(),
                                v_out=v_new.data_ptr(), workspace=work.data_ptr(), workspace_bytes=work.numel(),
                                weights_constant=1)
        if fused:
            dsc.kv_k_cache, dsc.kv_k_scale, dsc.kv_v_cache, dsc.kv_v_scale = [t.data_ptr() for t in fused]
            dsc.kv_capacity = capacity
        return dsc

    s = torch.cuda.current_stream().cuda_stream
    ka, ksa, va, vsa = caches()
    check(L.sb_linear_ex(ctypes.byref(desc(q_a, None)), s), "qkv")
    check(L.sb_kv_append_int8(k_new.data_ptr(), v_new.data_ptr(), ka.data_ptr(), ksa.data_ptr(), va.data_ptr(),
                              vsa.data_ptr(), bsz, hkv, 1, d, capacity, positions.data_ptr(), s), "kv_append")
    kb, ksb, vb, vsb = caches()
    check(L.sb_linear_ex(ctypes.byref(desc(q_b, (kb, ksb, vb, vsb))), s), "qkv fused")
    torch.cuda.synchronize()
    assert torch.equal(q_a, q_b)
    for a, b in ((ka, kb), (ksa, ksb), (va, vb), (vsa, vsb)):
        assert torch.equal(a, b)
    # the rows at the positions were written (not the fill values)
    assert not torch.equal(kb[0, :, int(positions[0])], torch.full_like(kb[0, :, 0], 3))
