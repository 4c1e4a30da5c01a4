"""Kernel parity on the GPU, through the C ABI, against the reference's golden
outputs and the CPU oracle.

Tolerances: packing is bit-exact; fp32 linear / attention outputs are
compared with a relative L2 error (the reference's own metric,
test_chunked_prefill.py:18-19) of at most 1e-5, and an element bound.
"""

import numpy as np
import pytest
import torch

import cases
from oracle import attention as oa
from oracle import model as om
from oracle import quant as oq

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-12))


def test_pack_bit_exact_vs_reference(golden):
    from kshipra_b200.quantization import quantize_int4_per_group, quantize_int8_per_channel
    g = golden("quant.npz")
    for name, w, scheme, gs in cases.quant_cases():
        if scheme == "int8":
            qw = quantize_int8_per_channel(w.cuda())
        else:
            qw = quantize_int4_per_group(w.cuda(), gs)
            assert qw.in_features_padded == (w.shape[1] + gs - 1) // gs * gs
        np.testing.assert_array_equal(qw.payload.cpu().numpy(), g[f"{name}/payload"], err_msg=name)
        np.testing.assert_array_equal(qw.scales.cpu().numpy().view(np.uint16),
                                      g[f"{name}/scales"].view(np.uint16), err_msg=name)


def test_pack_large_matches_oracle():
    from kshipra_b200.quantization import quantize_int4_per_group, quantize_int8_per_channel
    gen = torch.Generator().manual_seed(123)
    w = torch.randn((1024, 4096), generator=gen) * 0.02
    w[3] = 0.0
    w[5, :128] = 1e-9
    q8 = quantize_int8_per_channel(w.cuda())
    p, s = oq.quantize_int8_per_channel(w.numpy())
    np.testing.assert_array_equal(q8.payload.cpu().numpy(), p)
    np.testing.assert_array_equal(q8.scales.cpu().numpy().view(np.uint16), s.view(np.uint16))
    q4 = quantize_int4_per_group(w.cuda(), 128)
    p, s, _ = oq.quantize_int4_per_group(w.numpy(), 128)
    np.testing.assert_array_equal(q4.payload.cpu().numpy(), p)
    np.testing.assert_array_equal(q4.scales.cpu().numpy().view(np.uint16), s.view(np.uint16))


def test_pack_rejects_nonfinite_and_bad_group():
    from kshipra_b200.quantization import (QuantizationError, quantize_int4_per_group,
                                           quantize_int8_per_channel)
    with pytest.raises(QuantizationError):
        quantize_int8_per_channel(torch.tensor([[1.0, float("nan")]], device="cuda"))
    with pytest.raises(QuantizationError):
        quantize_int4_per_group(torch.tensor([[1.0, float("inf")]], device="cuda"))
    with pytest.raises(QuantizationError):
        quantize_int4_per_group(torch.ones(4, 128, device="cuda"), 127)
    with pytest.raises(QuantizationError):
        quantize_int4_per_group(torch.ones(4, 128, device="cuda"), 0)


def test_quantized_linear_vs_reference(golden):
    import torch.nn as nn
    from kshipra_b200.quantization import QuantizedLinear
    g = golden("qlinear.npz")
    for name, x, w, b, scheme, gs in cases.qlinear_cases():
        lin = nn.Linear(w.shape[1], w.shape[0], bias=b is not None)
        with torch.no_grad():
            lin.weight.copy_(w)
            if b is not None:
                lin.bias.copy_(b)
        ql = QuantizedLinear(lin, scheme=scheme, group_size=gs)
        y = ql(x.cuda()).cpu().numpy()
        ref = g[name]
        assert rel_l2(y, ref) < 1e-5, (name, rel_l2(y, ref))
        # exact-math check: fp64 product with the oracle's dequantized weight
        wn = w.numpy()
        if scheme == "int8":
            p, s = oq.quantize_int8_per_channel(wn)
            wd = oq.dequantize_int8(p, s)
        else:
            p, s, _ = oq.quantize_int4_per_group(wn, gs)
            wd = oq.dequantize_int4(p, s, wn.shape[1], gs)
        y64 = x.numpy().astype(np.float64) @ wd.astype(np.float64).T
        if b is not None:
            y64 += b.numpy()
        assert np.abs(y - y64).max() <= 1e-5 * max(np.abs(y64).max(), 1.0), name


@pytest.mark.parametrize("scheme", ["int8", "int4", "fp32"])
@pytest.mark.parametrize("m", [1, 2, 5, 8, 16, 17, 64, 200])
def test_linear_paths_residual_and_swiglu(scheme, m):
    """GEMV (m <= 16) and GEMM paths, residual add and SwiGLU fusion."""
    from kshipra_b200.quantization import (linear_launch, quantize_int4_per_group,
                                           quantize_int8_per_channel, swiglu_launch)
    gen = torch.Generator().manual_seed(m)
    K, N, I = 896, 1152, 640
    x = torch.randn((m, K), generator=gen)
    w = torch.randn((N, K), generator=gen) * 0.03
    wgu = torch.randn((2 * I, K), generator=gen) * 0.03
    res = torch.randn((m, N), generator=gen)
    bias = torch.randn((N,), generator=gen)
    if scheme == "int8":
        qw, qgu = quantize_int8_per_channel(w.cuda()), quantize_int8_per_channel(wgu.cuda())
        wd = oq.dequantize_int8(*oq.quantize_int8_per_channel(w.numpy()))
        gud = oq.dequantize_int8(*oq.quantize_int8_per_channel(wgu.numpy()))
        wf = gf = None
    elif scheme == "int4":
        qw, qgu = quantize_int4_per_group(w.cuda()), quantize_int4_per_group(wgu.cuda())
        p, s, _ = oq.quantize_int4_per_group(w.numpy(), 128)
        wd = oq.dequantize_int4(p, s, K, 128)
        p, s, _ = oq.quantize_int4_per_group(wgu.numpy(), 128)
        gud = oq.dequantize_int4(p, s, K, 128)
        wf = gf = None
    else:
        qw = qgu = None
        wf, gf = w.cuda(), wgu.cuda()
        wd, gud = w.numpy(), wgu.numpy()
    from kshipra_b200 import _lib
    xc = x.cuda()
    y64 = x.double().numpy() @ wd.astype(np.float64).T + bias.double().numpy() + res.double().numpy()
    gu = x.double().numpy() @ gud.astype(np.float64).T
    gg, uu = gu[:, :I], gu[:, I:]
    h64 = gg / (1 + np.exp(-gg)) * uu
    # both decode GEMV variants (register-resident and streaming) for small m
    for resident in (1, 0):
        prev = _lib.lib().ksh_set_gemv_resident(resident)
        try:
            y = res.clone().cuda()
            linear_launch(xc, qw, wf, bias.cuda(), y, residual=y)
            assert np.abs(y.cpu().numpy() - y64).max() <= 2e-5 * np.abs(y64).max(), resident
            h = torch.empty((m, I), device="cuda")
            swiglu_launch(xc, qgu, gf, I, h)
            assert np.abs(h.cpu().numpy() - h64).max() <= 2e-5 * max(np.abs(h64).max(), 1.0), resident
        finally:
            _lib.lib().ksh_set_gemv_resident(prev)


def _rms_norm64(x, nw, eps=1e-6):
    x = x.astype(np.float64)
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * nw.astype(np.float64)


@pytest.mark.parametrize("scheme", ["int8", "int4"])
@pytest.mark.parametrize("m", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("K,N,I", [(896, 1152, 640), (912, 1000, 328), (4096, 6144, 1536)])
def test_tensor_core_decode_linear(scheme, m, K, N, I):
    """Swap-AB tcgen05 decode path (forced for every shape) against fp64 with
    the dequantized weight: bias + residual, fused RMSNorm, SwiGLU; tiles that
    overhang N, K not a multiple of the 64-wide stage."""
    from kshipra_b200 import _lib
    from kshipra_b200.quantization import (linear_launch, quantize_int4_per_group,
                                           quantize_int8_per_channel, swiglu_launch)
    gen = torch.Generator().manual_seed(m * 31 + K + N)
    x = torch.randn((m, K), generator=gen)
    x[0] *= 40.0                               # token rows of very different size
    w = torch.randn((N, K), generator=gen) * 0.03
    wgu = torch.randn((2 * I, K), generator=gen) * 0.03
    res = torch.randn((m, N), generator=gen)
    bias = torch.randn((N,), generator=gen)
    nw = 1.0 + 0.2 * torch.randn((K,), generator=gen)
    if scheme == "int8":
        qw, qgu = quantize_int8_per_channel(w.cuda()), quantize_int8_per_channel(wgu.cuda())
        wd = oq.dequantize_int8(*oq.quantize_int8_per_channel(w.numpy()))
        gud = oq.dequantize_int8(*oq.quantize_int8_per_channel(wgu.numpy()))
    else:
        qw, qgu = quantize_int4_per_group(w.cuda()), quantize_int4_per_group(wgu.cuda())
        p, s, _ = oq.quantize_int4_per_group(w.numpy(), 128)
        wd = oq.dequantize_int4(p, s, K, 128)
        p, s, _ = oq.quantize_int4_per_group(wgu.numpy(), 128)
        gud = oq.dequantize_int4(p, s, K, 128)
    wd, gud = wd.astype(np.float64), gud.astype(np.float64)
    x64 = x.double().numpy()
    xn64 = _rms_norm64(x.numpy(), nw.numpy())
    y64 = x64 @ wd.T + bias.double().numpy() + res.double().numpy()
    yn64 = xn64 @ wd.T
    gu = xn64 @ gud.T
    h64 = gu[:, :I] / (1 + np.exp(-gu[:, :I])) * gu[:, I:]
    xc, nc = x.cuda(), nw.cuda()
    modes = (2, 3)       # integer-MMA kernels, then the fp16-operand kernel
    prev = _lib.lib().ksh_set_gemv_tc(2)
    prev_dp4a = _lib.lib().ksh_set_gemv_dp4a(0)     # one-row INT4 would take the dp4a kernel
    try:
        for mode in modes:
            _lib.lib().ksh_set_gemv_tc(mode)
            for _ in range(2):
                y = res.clone().cuda()
                linear_launch(xc, qw, None, bias.cuda(), y, residual=y)
                err = np.abs(y.cpu().numpy() - y64).max(axis=1) / np.abs(y64).max(axis=1)
                assert err.max() <= 2e-5, (mode, err)
                yn = torch.empty((m, N), device="cuda")
                linear_launch(xc, qw, None, None, yn, norm_w=nc)
                err = np.abs(yn.cpu().numpy() - yn64).max(axis=1) / np.abs(yn64).max(axis=1)
                assert err.max() <= 2e-5, (mode, err)
                h = torch.empty((m, I), device="cuda")
                swiglu_launch(xc, qgu, None, I, h, norm_w=nc)
                err = np.abs(h.cpu().numpy() - h64).max(axis=1) / np.maximum(np.abs(h64).max(axis=1), 1e-3)
                assert err.max() <= 2e-5, (mode, err)
    finally:
        _lib.lib().ksh_set_gemv_tc(prev)
        _lib.lib().ksh_set_gemv_dp4a(prev_dp4a)


@pytest.mark.parametrize("scheme,g", [("int8", 0), ("int4", 128), ("int4", 64)])
@pytest.mark.parametrize("m", [17, 31, 32, 33, 48, 64])
@pytest.mark.parametrize("K,N,I", [(896, 1152, 640), (912, 1000, 328), (4096, 6144, 1536)])
def test_mid_batch_linear(scheme, g, m, K, N, I):
    """17..64 token rows through the swap-AB tensor-core kernel, then through
    the prefill GEMM (kernel switched off), each against fp64 with the
    dequantized weight: bias + residual, fused RMSNorm, SwiGLU; tiles that
    overhang N, K not a multiple of the 64-wide stage, rows of very different
    size."""
    from kshipra_b200 import _lib
    from kshipra_b200.quantization import (linear_launch, quantize_int4_per_group,
                                           quantize_int8_per_channel, swiglu_launch)
    gen = torch.Generator().manual_seed(m * 7 + K + N + g)
    x = torch.randn((m, K), generator=gen)
    x[0] *= 40.0
    x[m - 1] *= 1e-3
    w = torch.randn((N, K), generator=gen) * 0.03
    wgu = torch.randn((2 * I, K), generator=gen) * 0.03
    res = torch.randn((m, N), generator=gen)
    bias = torch.randn((N,), generator=gen)
    nw = 1.0 + 0.2 * torch.randn((K,), generator=gen)
    if scheme == "int8":
        qw, qgu = quantize_int8_per_channel(w.cuda()), quantize_int8_per_channel(wgu.cuda())
        wd = oq.dequantize_int8(*oq.quantize_int8_per_channel(w.numpy()))
        gud = oq.dequantize_int8(*oq.quantize_int8_per_channel(wgu.numpy()))
    else:
        qw, qgu = quantize_int4_per_group(w.cuda(), g), quantize_int4_per_group(wgu.cuda(), g)
        p, s, _ = oq.quantize_int4_per_group(w.numpy(), g)
        wd = oq.dequantize_int4(p, s, K, g)
        p, s, _ = oq.quantize_int4_per_group(wgu.numpy(), g)
        gud = oq.dequantize_int4(p, s, K, g)
    wd, gud = wd.astype(np.float64), gud.astype(np.float64)
    x64 = x.double().numpy()
    xn64 = _rms_norm64(x.numpy(), nw.numpy())
    y64 = x64 @ wd.T + bias.double().numpy() + res.double().numpy()
    yn64 = xn64 @ wd.T
    gu = xn64 @ gud.T
    h64 = gu[:, :I] / (1 + np.exp(-gu[:, :I])) * gu[:, I:]
    xc, nc = x.cuda(), nw.cuda()
    prev = _lib.lib().ksh_set_gemm_mid(1)
    try:
        for mode in (1, 0):
            _lib.lib().ksh_set_gemm_mid(mode)
            for _ in range(2):
                y = res.clone().cuda()
                n0 = _lib.lib().ksh_kernel_launches()
                linear_launch(xc, qw, None, bias.cuda(), y, residual=y)
                assert _lib.lib().ksh_kernel_launches() - n0 == 2     # x split + GEMM
                err = np.abs(y.cpu().numpy() - y64).max(axis=1) / np.abs(y64).max(axis=1)
                assert err.max() <= 2e-5, (mode, err)
                yn = torch.empty((m, N), device="cuda")
                linear_launch(xc, qw, None, None, yn, norm_w=nc)
                err = np.abs(yn.cpu().numpy() - yn64).max(axis=1) / np.abs(yn64).max(axis=1)
                assert err.max() <= 2e-5, (mode, err)
                h = torch.empty((m, I), device="cuda")
                swiglu_launch(xc, qgu, None, I, h, norm_w=nc)
                err = np.abs(h.cpu().numpy() - h64).max(axis=1) / np.maximum(np.abs(h64).max(axis=1), 1e-3)
                assert err.max() <= 2e-5, (mode, err)
    finally:
        _lib.lib().ksh_set_gemm_mid(prev)


@pytest.mark.parametrize("g", [32, 64, 128])
@pytest.mark.parametrize("K,N,I", [(896, 1152, 640), (912, 999, 328), (4096, 6144, 1536),
                                   (14336, 512, 64)])
def test_dp4a_one_row_int4_linear(g, K, N, I):
    """One-row INT4 linears through the dp4a kernel against fp64 with the
    dequantized weight: bias + residual, fused RMSNorm, SwiGLU; an odd row
    count (the last row pair has one row), K not a multiple of the group."""
    from kshipra_b200 import _lib
    from kshipra_b200.quantization import linear_launch, quantize_int4_per_group, swiglu_launch
    gen = torch.Generator().manual_seed(g + K + N)
    x = torch.randn((1, K), generator=gen) * 3.0
    x[0, ::7] *= 1e-3                          # entries of very different size in one vector
    w = torch.randn((N, K), generator=gen) * 0.03
    wgu = torch.randn((2 * I, K), generator=gen) * 0.03
    res = torch.randn((1, N), generator=gen)
    bias = torch.randn((N,), generator=gen)
    nw = 1.0 + 0.2 * torch.randn((K,), generator=gen)
    qw, qgu = quantize_int4_per_group(w.cuda(), g), quantize_int4_per_group(wgu.cuda(), g)
    p, s, _ = oq.quantize_int4_per_group(w.numpy(), g)
    wd = oq.dequantize_int4(p, s, K, g).astype(np.float64)
    p, s, _ = oq.quantize_int4_per_group(wgu.numpy(), g)
    gud = oq.dequantize_int4(p, s, K, g).astype(np.float64)
    x64 = x.double().numpy()
    xn64 = _rms_norm64(x.numpy(), nw.numpy())
    y64 = x64 @ wd.T + bias.double().numpy() + res.double().numpy()
    yn64 = xn64 @ wd.T
    gu = xn64 @ gud.T
    h64 = gu[:, :I] / (1 + np.exp(-gu[:, :I])) * gu[:, I:]
    xc, nc = x.cuda(), nw.cuda()
    prev = _lib.lib().ksh_set_gemv_dp4a(1)
    try:
        n0 = _lib.lib().ksh_kernel_launches()
        y = res.clone().cuda()
        linear_launch(xc, qw, None, bias.cuda(), y, residual=y)
        assert _lib.lib().ksh_kernel_launches() - n0 == 1
        err = np.abs(y.cpu().numpy() - y64).max() / np.abs(y64).max()
        assert err <= 2e-6, err
        yn = torch.empty((1, N), device="cuda")
        linear_launch(xc, qw, None, None, yn, norm_w=nc)
        err = np.abs(yn.cpu().numpy() - yn64).max() / np.abs(yn64).max()
        assert err <= 2e-6, err
        h = torch.empty((1, I), device="cuda")
        swiglu_launch(xc, qgu, None, I, h, norm_w=nc)
        err = np.abs(h.cpu().numpy() - h64).max() / max(np.abs(h64).max(), 1e-3)
        assert err <= 2e-6, err
    finally:
        _lib.lib().ksh_set_gemv_dp4a(prev)


def _run_attention_case(q, kp, vp, bt, P, C, B):
    from kshipra_b200.chunked_prefill import chunked_attention
    return chunked_attention(q.cuda(), kp.cuda(), vp.cuda(), bt, P, C, B).cpu()


def test_attention_vs_reference(golden):
    g = golden("attention.npz")
    for c in cases.attention_cases():
        q, kp, vp, bt = cases.attention_inputs(c)
        out = _run_attention_case(q, kp, vp, bt, c["P"], c["C"], c["B"]).numpy()
        ref = g[c["name"]]
        assert rel_l2(out, ref) < 1e-5, (c["name"], rel_l2(out, ref))
        assert np.abs(out - ref).max() < 1e-4, c["name"]
    q, kp, vp, bt, P, C, B = cases.mask_kat_inputs()
    out = _run_attention_case(q, kp, vp, bt, P, C, B).numpy()
    np.testing.assert_allclose(out, g["mask_kat"], atol=1e-5)


def test_attention_pool_view_and_batched_varlen():
    """In-place pool views and a varlen batch (decode + prefill rows mixed)."""
    from kshipra_b200.chunked_prefill import chunked_attention, paged_attention
    gen = torch.Generator().manual_seed(5)
    nb, L, hkv, B, D, hq = 40, 3, 2, 16, 64, 14
    pool = torch.randn((nb, L, 2, hkv, B, D), generator=gen)
    layer = 1
    seqs = [(0, 37, 1), (1, 100, 5), (2, 0, 20), (3, 63, 1), (4, 200, 33)]
    perm = torch.randperm(nb, generator=gen).tolist()
    tables, starts, pls, qs = [], [0], [], []
    off = 0
    for i, (_, P, C) in enumerate(seqs):
        nblk = (P + C + B - 1) // B
        tables.append(perm[off:off + nblk])
        off += nblk
        starts.append(starts[-1] + C)
        pls.append(P)
        qs.append(torch.randn((hq, C, D), generator=gen))
    maxb = max(len(t) for t in tables)
    bt = torch.zeros((len(seqs), maxb), dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t)
    qcat = torch.cat([q.transpose(0, 1) for q in qs], dim=0).contiguous()
    out = torch.empty_like(qcat).cuda()
    poolc = pool.cuda()
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    paged_attention(qcat.cuda(), poolc, layer, bt.cuda(), torch.tensor(starts, dtype=torch.int32).cuda(),
                    torch.tensor(pls, dtype=torch.int32).cuda(), max(c for _, _, c in seqs),
                    max(p + c for _, p, c in seqs), out, flags)
    assert int(flags.item()) == 0
    out = out.cpu()
    for i, (_, P, C) in enumerate(seqs):
        ref = oa.chunked_attention(qs[i], pool[:, layer, 0], pool[:, layer, 1], tables[i], P, C, B)
        got = out[starts[i]:starts[i + 1]].transpose(0, 1)
        assert rel_l2(got.numpy(), ref.numpy()) < 1e-5, i
        # the drop-in API reading the pool views in place
        got2 = chunked_attention(qs[i].cuda(), poolc[:, layer, 0], poolc[:, layer, 1], tables[i],
                                 P, C, B).cpu()
        assert rel_l2(got2.numpy(), ref.numpy()) < 1e-5, i


def test_attention_bad_block_id_flags():
    from kshipra_b200.chunked_prefill import chunked_attention
    q = torch.randn(4, 1, 64)
    kp = torch.randn(4, 2, 16, 64)
    with pytest.raises(IndexError):
        chunked_attention(q.cuda(), kp.cuda(), kp.cuda(), [0, 99], 20, 1, 16)


def test_rmsnorm_rope_kv_vs_oracle():
    from kshipra_b200 import _lib
    from kshipra_b200.model import rope_tables
    gen = torch.Generator().manual_seed(3)
    T, H, hq, hkv, D = 7, 896, 14, 2, 64
    x = torch.randn((T, H), generator=gen) * 3
    w = torch.randn((H,), generator=gen)
    y = torch.empty((T, H), device="cuda")
    xc, wc = x.cuda(), w.cuda()      # keep device copies alive across the launch
    _lib.call("ksh_rmsnorm", xc.data_ptr(), wc.data_ptr(), y.data_ptr(), T, H, 1e-6,
              _lib.stream_ptr())
    ref = om.rms_norm(x, w, 1e-6)
    assert np.abs(y.cpu().numpy() - ref.numpy()).max() <= 1e-6 * np.abs(ref.numpy()).max()
    # RoPE + scatter
    theta, maxp = 1e6, 4096
    rc, rs = rope_tables(D, theta, maxp)
    qkv = torch.randn((T, (hq + 2 * hkv) * D), generator=gen)
    pos = torch.tensor([0, 1, 5, 17, 100, 2047, 4095])
    nb, L, B = 300, 2, 16
    slots = torch.randperm(nb * B, generator=gen)[:T]
    pool = torch.zeros((nb, L, 2, hkv, B, D), device="cuda")
    qo = torch.empty((T, hq, D), device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    dev = [t.cuda() for t in (qkv, pos, slots, rc, rs)]
    _lib.call("ksh_rope_kv_write", dev[0].data_ptr(), T, hq, hkv, D, dev[1].data_ptr(),
              dev[2].data_ptr(), dev[3].data_ptr(), dev[4].data_ptr(), maxp,
              qo.data_ptr(), pool.data_ptr(), nb, L, 1, B, flags.data_ptr(), _lib.stream_ptr())
    assert int(flags.item()) == 0
    cos, sin = om.compute_rope(D, pos.unsqueeze(0), theta)
    q = qkv[:, :hq * D].view(1, T, hq, D).transpose(1, 2)
    k = qkv[:, hq * D:(hq + hkv) * D].view(1, T, hkv, D).transpose(1, 2)
    v = qkv[:, (hq + hkv) * D:].view(T, hkv, D)
    qr, kr = om.apply_rope(q, k, cos, sin)
    np.testing.assert_array_equal(qo.cpu().numpy(), qr[0].transpose(0, 1).numpy())
    pc = pool.cpu()
    for t in range(T):
        s = int(slots[t])
        np.testing.assert_array_equal(pc[s // B, 1, 0, :, s % B].numpy(), kr[0, :, t].numpy())
        np.testing.assert_array_equal(pc[s // B, 1, 1, :, s % B].numpy(), v[t].numpy())
    assert float(pc[:, 0].abs().sum()) == 0.0


def test_lm_head_argmax_first_index():
    from kshipra_b200 import _lib
    gen = torch.Generator().manual_seed(9)
    V, H = 151936, 896
    w = torch.randn((V, H), generator=gen) * 0.02
    w[77] = w[151000]          # exact tie: the lower index must win
    for m in (1, 3, 16, 20):
        x = torch.randn((m, H), generator=gen)
        x[0] = w[151000] * 50
        logits = torch.empty((m, V), device="cuda")
        tok = torch.empty(m, dtype=torch.int64, device="cuda")
        ws = torch.zeros(int(_lib.lib().ksh_lm_head_workspace_size(m, V)), dtype=torch.uint8,
                         device="cuda")
        wc, xc = w.cuda(), x.cuda()
        _lib.call("ksh_lm_head_argmax", xc.data_ptr(), m, H, None, 0.0, wc.data_ptr(), V,
                  logits.data_ptr(), tok.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        ref = x.double() @ w.double().T
        lg = logits.cpu()
        assert float((lg.double() - ref).abs().max()) <= 1e-5 * float(ref.abs().max())
        assert tok.cpu().tolist() == torch.argmax(lg, dim=1).tolist()
        assert int(tok[0]) == 77
        # argmax-only call (no logits) agrees, and a logits-only call
        tok2 = torch.empty(m, dtype=torch.int64, device="cuda")
        _lib.call("ksh_lm_head_argmax", xc.data_ptr(), m, H, None, 0.0, wc.data_ptr(), V, None,
                  tok2.data_ptr(), ws.data_ptr(), ws.numel(), _lib.stream_ptr())
        assert tok2.cpu().tolist() == tok.cpu().tolist()
        if m > 16:
            lg2 = torch.empty((m, V), device="cuda")
            _lib.call("ksh_lm_head_argmax", xc.data_ptr(), m, H, None, 0.0, wc.data_ptr(), V,
                      lg2.data_ptr(), None, ws.data_ptr(), ws.numel(), _lib.stream_ptr())
            assert torch.equal(lg2.cpu(), lg)


@pytest.mark.parametrize("m,H,V", [(8, 4096, 128256), (16, 2048, 32000), (5, 4096, 1000),
                                   (17, 4096, 128256), (64, 4096, 128256), (100, 896, 1000),
                                   (33, 900, 130)])
def test_lm_head_argmax_tiled_x_stays_in_workspace(m, H, V):
    """Hidden sizes whose staged activations span several shared-memory tiles
    (Llama-3-8B lm_head at batch 5-16), and the batch path above 16 rows
    (64 rows per launch, ragged vocabulary tiles, a hidden size that is not a
    multiple of the 32-float weight step): logits, first-index argmax, and no
    write past the workspace the size query asked for."""
    from kshipra_b200 import _lib
    gen = torch.Generator().manual_seed(m + H + V)
    w = torch.randn((V, H), generator=gen) * 0.02
    w[V // 3] = w[V - 5]
    x = torch.randn((m, H), generator=gen)
    x[0] = w[V - 5] * 50
    nw = 1.0 + 0.1 * torch.randn(H, generator=gen)
    wc, xc, nc = w.cuda(), x.cuda(), nw.cuda()
    need = int(_lib.lib().ksh_lm_head_workspace_size(m, V))
    guard = 1 << 20
    ws = torch.zeros(need + guard, dtype=torch.uint8, device="cuda")
    ws[need:] = 0xAB
    logits = torch.empty((m, V), device="cuda")
    tok = torch.empty(m, dtype=torch.int64, device="cuda")
    for _ in range(2):
        _lib.call("ksh_lm_head_argmax", xc.data_ptr(), m, H, nc.data_ptr(), 1e-6, wc.data_ptr(),
                  V, logits.data_ptr(), tok.data_ptr(), ws.data_ptr(), need, _lib.stream_ptr())
        torch.cuda.synchronize()
        assert bool((ws[need:] == 0xAB).all())
        xd = x.double()
        xn = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.double()
        ref = xn @ w.double().T
        lg = logits.cpu()
        assert float((lg.double() - ref).abs().max()) <= 1e-5 * float(ref.abs().max())
        assert tok.cpu().tolist() == torch.argmax(lg, dim=1).tolist()
        assert int(tok[0]) == V // 3


@pytest.mark.parametrize("m", [1, 16, 40])
def test_lm_head_argmax_accepts_uninitialised_workspace(m):
    """A workspace straight from the allocator (here filled with 0xFF bytes)
    is valid: the entry point clears its completion counter before the
    kernels run, for the GEMV path (<= 16 rows) and the batch path."""
    from kshipra_b200 import _lib
    gen = torch.Generator().manual_seed(40 + m)
    V, H = 50000, 1024
    w = (torch.randn((V, H), generator=gen) * 0.02).cuda()
    x = torch.randn((m, H), generator=gen).cuda()
    need = int(_lib.lib().ksh_lm_head_workspace_size(m, V))
    out = {}
    for fill in (0x00, 0xFF):
        ws = torch.full((need,), fill, dtype=torch.uint8, device="cuda")
        lg = torch.empty((m, V), device="cuda")
        tok = torch.full((m,), -1, dtype=torch.int64, device="cuda")
        for _ in range(2):
            _lib.call("ksh_lm_head_argmax", x.data_ptr(), m, H, None, 0.0, w.data_ptr(), V,
                      lg.data_ptr(), tok.data_ptr(), ws.data_ptr(), need, _lib.stream_ptr())
            torch.cuda.synchronize()
            out.setdefault(fill, []).append((tok.cpu().tolist(), lg.cpu()))
    ref = torch.argmax(out[0][0][1], dim=1).tolist()
    for fill in (0x00, 0xFF):
        for toks, lg in out[fill]:
            assert toks == ref, fill
            assert torch.equal(lg, out[0][0][1])


def test_paged_attention_accepts_uninitialised_workspace():
    """Split-K attention with its counters in a 0xFF-filled workspace gives
    the result of a zeroed one (the entry point clears the counters)."""
    from kshipra_b200.chunked_prefill import AttentionWorkspace, paged_attention
    gen = torch.Generator().manual_seed(3)
    nb, L, hkv, B, D, hq = 80, 2, 2, 16, 64, 14
    pool = torch.randn((nb, L, 2, hkv, B, D), generator=gen).cuda()
    P, C = 700, 3
    nblk = (P + C + B - 1) // B
    bt = torch.arange(nblk, dtype=torch.int32).view(1, -1).cuda()
    q = torch.randn((C, hq, D), generator=gen).cuda()
    qs = torch.tensor([0, C], dtype=torch.int32).cuda()
    pl = torch.tensor([P], dtype=torch.int32).cuda()
    res = []
    for fill in (0x00, 0xFF):
        ws = AttentionWorkspace()
        ws.buf = torch.full((1 << 22,), fill, dtype=torch.uint8, device="cuda")
        out = torch.empty_like(q)
        flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        for _ in range(2):
            paged_attention(q, pool, 1, bt, qs, pl, C, P + C, out, flags, ws=ws)
            res.append(out.cpu().clone())
        assert int(flags.item()) == 0
    ref = oa.chunked_attention(q.cpu().transpose(0, 1), pool.cpu()[:, 1, 0], pool.cpu()[:, 1, 1],
                               list(range(nblk)), P, C, B).transpose(0, 1)
    for r in res:
        assert torch.equal(r, res[0])
    assert rel_l2(res[0].numpy(), ref.numpy()) < 1e-5


@pytest.mark.parametrize("scheme", ["int8", "int4"])
@pytest.mark.parametrize("m,k,n", [(128, 896, 1152), (512, 4864, 896), (130, 896, 9728),
                                   (2048, 4096, 512)])
def test_tensor_core_gemm_prefill_shapes(scheme, m, k, n):
    """tcgen05 path at the prefill shapes: fp64 reference with the dequantized weight."""
    from kshipra_b200.quantization import (linear_launch, quantize_int4_per_group,
                                           quantize_int8_per_channel, swiglu_launch)
    gen = torch.Generator().manual_seed(m + k + n)
    x = torch.randn((m, k), generator=gen)
    x[3] *= 1e-3                        # rows with very different magnitudes
    x[5] *= 300.0
    w = torch.randn((n, k), generator=gen) * 0.02
    if scheme == "int8":
        qw = quantize_int8_per_channel(w.cuda())
        wd = oq.dequantize_int8(qw.payload.cpu().numpy(), qw.scales.cpu().numpy())
    else:
        qw = quantize_int4_per_group(w.cuda(), 128)
        wd = oq.dequantize_int4(qw.payload.cpu().numpy(), qw.scales.cpu().numpy(), k, 128)
    y = torch.empty((m, n), device="cuda")
    linear_launch(x.cuda(), qw, None, None, y)
    y64 = x.double().numpy() @ wd.astype(np.float64).T
    err = np.abs(y.cpu().numpy() - y64) / (np.abs(x.double().numpy()).max(axis=1, keepdims=True)
                                           * np.abs(wd).max() * np.sqrt(k))
    assert err.max() < 1e-6, err.max()
    if n % 2 == 0:
        inter = n // 2
        h = torch.empty((m, inter), device="cuda")
        swiglu_launch(x.cuda(), qw, None, inter, h)
        g, u = y64[:, :inter], y64[:, inter:]
        h64 = g / (1 + np.exp(-g)) * u
        assert np.abs(h.cpu().numpy() - h64).max() <= 1e-5 * max(np.abs(h64).max(), 1.0)


@pytest.mark.parametrize("D,hq,hkv,bs", [(64, 14, 2, 16), (64, 4, 2, 32), (128, 32, 8, 16),
                                         (128, 8, 8, 64), (64, 8, 1, 16)])
def test_fused_decode_attention_vs_oracle(D, hq, hkv, bs):
    """RoPE + K/V write + attention of one new token per sequence, batched."""
    from kshipra_b200 import _lib
    from kshipra_b200.model import rope_tables
    gen = torch.Generator().manual_seed(D + hq + bs)
    positions = [0, 5, 15, 16, 100, 561, 1023, 3000]
    B = len(positions)
    L, layer = 2, 1
    maxb = (max(positions) + 1 + bs - 1) // bs + 1
    nb = B * maxb + 3
    perm = torch.randperm(nb, generator=gen)
    bt = perm[:B * maxb].view(B, maxb).to(torch.int32)
    pool = torch.randn((nb, L, 2, hkv, bs, D), generator=gen)
    qkv = torch.randn((B, (hq + 2 * hkv) * D), generator=gen)
    rc, rs = rope_tables(D, 10000.0, 4096)
    pos = torch.tensor(positions, dtype=torch.int64)
    slots = torch.tensor([int(bt[b, p // bs]) * bs + p % bs for b, p in enumerate(positions)])
    dev = [t.cuda() for t in (qkv, pos, slots, rc, rs, bt)]
    poolc = pool.cuda()
    outs = {}
    # every key split (CTAs per sequence and kv head), and the per-launch choice (0)
    for split in (0, 1, 2, 3, 5, 8):
        out = torch.empty((B, hq, D), device="cuda")
        flags = torch.zeros(1, dtype=torch.int32, device="cuda")
        prev = _lib.lib().ksh_set_decode_split(split)
        try:
            _lib.call("ksh_decode_attention", dev[0].data_ptr(), B, hq, hkv, D, dev[1].data_ptr(),
                      dev[2].data_ptr(), dev[3].data_ptr(), dev[4].data_ptr(), 4096,
                      poolc.data_ptr(), nb, L, layer, bs, dev[5].data_ptr(), maxb,
                      max(positions) + 1, out.data_ptr(), flags.data_ptr(), _lib.stream_ptr())
        finally:
            _lib.lib().ksh_set_decode_split(prev)
        assert int(flags.item()) == 0, split
        outs[split] = out.cpu()
    pool_after = poolc.cpu()
    ref_pool = pool          # block tables are disjoint: one reference pool serves all
    qrs = []
    for b, p in enumerate(positions):
        cos, sin = om.compute_rope(D, torch.tensor([[p]]), 10000.0)
        q = qkv[b, :hq * D].view(1, 1, hq, D).transpose(1, 2)
        k = qkv[b, hq * D:(hq + hkv) * D].view(1, 1, hkv, D).transpose(1, 2)
        v = qkv[b, (hq + hkv) * D:].view(hkv, D)
        qr, kr = om.apply_rope(q, k, cos, sin)
        qrs.append(qr)
        s = int(slots[b])
        ref_pool[s // bs, layer, 0, :, s % bs] = kr[0, :, 0]
        ref_pool[s // bs, layer, 1, :, s % bs] = v
        np.testing.assert_array_equal(pool_after[s // bs, layer, :, :, s % bs].numpy(),
                                      ref_pool[s // bs, layer, :, :, s % bs].numpy())
    for b, p in enumerate(positions):
        qr = qrs[b]
        ref = oa.chunked_attention(qr[0], ref_pool[:, layer, 0], ref_pool[:, layer, 1],
                                   bt[b].tolist(), p, 1, bs)
        for split, out in outs.items():
            got = out[b].unsqueeze(1)
            err = rel_l2(got.numpy(), ref.numpy())
            assert err < 1e-5, (split, b, p, err)


def test_fused_decode_attention_shared_prefix_blocks():
    """Block tables that share their first blocks (a radix-cached prefix, as
    in the shared-prefix microbench): every sequence reads the same prefix
    blocks and writes its new token into its own block; outputs match a
    float64 torch reference of each sequence, at every key split."""
    from kshipra_b200 import _lib
    from kshipra_b200.model import rope_tables
    hq, hkv, D, bs = 32, 8, 128, 16
    g = hq // hkv
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(21)
    prefix_blocks = [3, 9, 0, 14]                      # 64 shared prefix positions
    suffix = [1, 37, 200]
    tables, positions, nxt = [], [], 20
    for s in suffix:
        own = list(range(nxt, nxt + (s + 1 + bs - 1) // bs))
        nxt += len(own)
        tables.append(prefix_blocks + own)
        positions.append(len(prefix_blocks) * bs + s)
    nb = nxt + 2
    maxb = max(len(t) for t in tables)
    bt = torch.full((len(tables), maxb), -1, dtype=torch.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    bt = bt.to(dev)
    B = len(tables)
    pool = torch.empty((nb, 1, 2, hkv, bs, D), device=dev).uniform_(-1.0, 1.0, generator=gen)
    qkv = torch.randn((B, (hq + 2 * hkv) * D), generator=gen, device=dev)
    rc, rs = (t.to(dev) for t in rope_tables(D, 500000.0, max(positions) + 1))
    pos = torch.tensor(positions, dtype=torch.int64, device=dev)
    slots = torch.tensor([tables[i][p // bs] * bs + p % bs for i, p in enumerate(positions)],
                         dtype=torch.int64, device=dev)
    prefix_before = pool[prefix_blocks].clone()
    half = D // 2
    for split in (0, 1, 4):
        out = torch.empty((B, hq, D), device=dev)
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        prev = _lib.lib().ksh_set_decode_split(split)
        try:
            _lib.call("ksh_decode_attention", qkv.data_ptr(), B, hq, hkv, D, pos.data_ptr(),
                      slots.data_ptr(), rc.data_ptr(), rs.data_ptr(), rc.shape[0], pool.data_ptr(),
                      nb, 1, 0, bs, bt.data_ptr(), maxb, max(positions) + 1, out.data_ptr(),
                      flags.data_ptr(), _lib.stream_ptr())
            torch.cuda.synchronize()
        finally:
            _lib.lib().ksh_set_decode_split(prev)
        assert int(flags.item()) == 0
        assert torch.equal(pool[prefix_blocks], prefix_before)      # the shared blocks stay intact
        for b, p in enumerate(positions):
            q = qkv[b, :hq * D].view(hq, D).double()
            c, s_ = rc[p].double(), rs[p].double()
            qr = torch.cat([q[:, :half] * c - q[:, half:] * s_, q[:, half:] * c + q[:, :half] * s_], 1)
            blk = torch.tensor([tables[b][t // bs] for t in range(p + 1)], device=dev)
            off = torch.tensor([t % bs for t in range(p + 1)], device=dev)
            K, V = pool[blk, 0, 0, :, off].double(), pool[blk, 0, 1, :, off].double()
            for hk in range(hkv):
                sc = qr[hk * g:(hk + 1) * g] @ K[:, hk].T / D ** 0.5
                ref = torch.softmax(sc, -1) @ V[:, hk]
                got = out[b, hk * g:(hk + 1) * g].double()
                assert float((got - ref).norm() / ref.norm()) < 1e-5, (split, b, hk)


def test_fused_decode_attention_long_context_batch64():
    """The 8B decode shape at full size: 64 sequences x 8 kv heads (g = 4,
    D = 128) at ragged lengths near 4096 keys over a 2 GB block pool, at the
    per-launch key split and at split 1 (the longest run of tiles per CTA).
    No flag may be raised (every stage wait completes), and sampled
    sequences match a float64 torch reference on the device."""
    from kshipra_b200 import _lib
    from kshipra_b200.model import rope_tables
    B, hq, hkv, D, bs, ctx = 64, 32, 8, 128, 16, 4096
    g = hq // hkv
    dev = torch.device("cuda")
    gen = torch.Generator(device=dev).manual_seed(11)
    positions = torch.tensor([ctx - (b * 37) % 300 for b in range(B)], dtype=torch.int64)
    maxb = (ctx + 1 + bs - 1) // bs
    nb = B * maxb
    bt = torch.randperm(nb, generator=torch.Generator().manual_seed(12)).view(B, maxb)
    bt = bt.to(torch.int32).to(dev)
    pool = torch.empty((nb, 1, 2, hkv, bs, D), device=dev).uniform_(-1.0, 1.0, generator=gen)
    qkv = torch.randn((B, (hq + 2 * hkv) * D), generator=gen, device=dev)
    rc, rs = (t.to(dev) for t in rope_tables(D, 500000.0, ctx + 1))
    pos = positions.to(dev)
    slots = torch.tensor([int(bt[b, int(p) // bs]) * bs + int(p) % bs
                          for b, p in enumerate(positions)], dtype=torch.int64, device=dev)
    outs = {}
    for split in (0, 1):
        out = torch.empty((B, hq, D), device=dev)
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        prev = _lib.lib().ksh_set_decode_split(split)
        try:
            _lib.call("ksh_decode_attention", qkv.data_ptr(), B, hq, hkv, D, pos.data_ptr(),
                      slots.data_ptr(), rc.data_ptr(), rs.data_ptr(), rc.shape[0],
                      pool.data_ptr(), nb, 1, 0, bs, bt.data_ptr(), maxb, ctx + 1,
                      out.data_ptr(), flags.data_ptr(), _lib.stream_ptr())
            torch.cuda.synchronize()
        finally:
            _lib.lib().ksh_set_decode_split(prev)
        assert int(flags.item()) == 0, (split, int(flags.item()))
        outs[split] = out
    # the workspace entry point: the cluster-free key split at the per-launch
    # choice and forced to 2..8 CTAs, each launch twice on one workspace (the
    # counters it leaves must serve the next launch)
    wsz = int(_lib.lib().ksh_decode_attention_workspace_size(B, hq, hkv, D))
    dws = torch.zeros(wsz, dtype=torch.uint8, device=dev)
    for gsplit in (0, 2, 3, 4, 5, 8):
        out = torch.empty((B, hq, D), device=dev)
        flags = torch.zeros(1, dtype=torch.int32, device=dev)
        prev = _lib.lib().ksh_set_decode_gsplit(gsplit)
        try:
            for _ in range(2):
                _lib.call("ksh_decode_attention_ws", qkv.data_ptr(), B, hq, hkv, D,
                          pos.data_ptr(), slots.data_ptr(), rc.data_ptr(), rs.data_ptr(),
                          rc.shape[0], pool.data_ptr(), nb, 1, 0, bs, bt.data_ptr(), maxb,
                          ctx + 1, out.data_ptr(), dws.data_ptr(), wsz, flags.data_ptr(),
                          _lib.stream_ptr())
            torch.cuda.synchronize()
        finally:
            _lib.lib().ksh_set_decode_gsplit(prev)
        assert int(flags.item()) == 0, (gsplit, int(flags.item()))
        outs[f"ws{gsplit}"] = out
    wsz_counters = (B * hkv * 4 + 255) // 256 * 256
    assert int(dws[:wsz_counters].sum()) == 0          # counters left at zero
    half = D // 2
    for b in (0, 9, 33, 63):
        p = int(positions[b])
        q = qkv[b, :hq * D].view(hq, D).double()
        c, s_ = rc[p].double(), rs[p].double()
        qr = torch.cat([q[:, :half] * c - q[:, half:] * s_, q[:, half:] * c + q[:, :half] * s_], 1)
        rows = [(int(bt[b, t // bs]), t % bs) for t in range(p + 1)]
        blk = torch.tensor([r[0] for r in rows], device=dev)
        off = torch.tensor([r[1] for r in rows], device=dev)
        K = pool[blk, 0, 0, :, off].double()            # [keys, hkv, D] (new row written by the call)
        V = pool[blk, 0, 1, :, off].double()
        for split, out in outs.items():
            for hk in range(hkv):
                sc = qr[hk * g:(hk + 1) * g] @ K[:, hk].T / D ** 0.5
                ref = torch.softmax(sc, -1) @ V[:, hk]
                got = out[b, hk * g:(hk + 1) * g].double()
                err = float((got - ref).norm() / ref.norm())
                assert err < 1e-5, (split, b, hk, err)


def test_chunked_prefill_engine_mock_layer_vs_cpu():
    """ChunkedPrefillEngine.prefill (chunked_prefill.py:148-246) with a mock
    one-layer model: each chunk's rotated K / V land in the pool at their
    slots (every layer of the pool, as the reference writes them), and the
    last chunk's attention over the whole prompt matches a float64 causal
    softmax on the CPU."""
    from kshipra_b200.chunked_prefill import ChunkedPrefillEngine
    from kshipra_b200.prefix_cache import PrefixCache
    gen = torch.Generator().manual_seed(21)
    V, H, HKV, D, B, P, CH = 500, 4, 2, 64, 16, 70, 16
    emb = torch.randn((V, 128), generator=gen)
    wq = torch.randn((128, H * D), generator=gen) * 0.1
    wk = torch.randn((128, HKV * D), generator=gen) * 0.1
    wv = torch.randn((128, HKV * D), generator=gen) * 0.1
    ids = torch.randint(0, V, (P,), generator=gen).tolist()
    cache = PrefixCache(num_blocks=12, block_size=B, num_layers=2, num_kv_heads=HKV, head_dim=D,
                        dtype=torch.float32, device=torch.device("cuda"))
    eng = ChunkedPrefillEngine(cache, chunk_size=CH, num_heads=H, num_kv_heads=HKV, head_dim=D)
    embc, wqc, wkc, wvc = emb.cuda(), wq.cuda(), wk.cuda(), wv.cuda()

    def rope(q, k, positions):
        c, s_ = om.compute_rope(D, positions.view(1, -1).cpu(), 10000.0)
        c, s_ = c[0].to(q.device), s_[0].to(q.device)
        rot = lambda x: x * c + om.rotate_half(x) * s_
        return rot(q), rot(k)

    def layer(x, attn_fn):
        q = (x @ wqc).view(-1, H, D).transpose(0, 1)
        k = (x @ wkc).view(-1, HKV, D).transpose(0, 1)
        v = (x @ wvc).view(-1, HKV, D).transpose(0, 1)
        return attn_fn(q.contiguous(), k.contiguous(), v.contiguous())

    taken = []
    orig_alloc = cache.allocate_blocks
    cache.allocate_blocks = lambda n: taken.extend(orig_alloc(n)) or taken[-n:]
    out = eng.prefill(ids, lambda t: embc[t], rope, layer)
    pool = cache.allocator.pool
    bt = list(taken)
    # reference: the whole prompt at once in float64 on the CPU
    x = emb[ids].double()
    pos = torch.arange(P)
    c, s_ = om.compute_rope(D, pos.view(1, -1), 10000.0)
    c, s_ = c[0].double(), s_[0].double()
    q = (x @ wq.double()).view(P, H, D).transpose(0, 1)
    k = (x @ wk.double()).view(P, HKV, D).transpose(0, 1)
    v = (x @ wv.double()).view(P, HKV, D).transpose(0, 1)
    q = q * c + om.rotate_half(q) * s_
    k = k * c + om.rotate_half(k) * s_
    last = P - (P - 1) // CH * CH
    qs = q[:, P - last:]
    kk = k.repeat_interleave(H // HKV, dim=0)
    vv = v.repeat_interleave(H // HKV, dim=0)
    sc = qs @ kk.transpose(1, 2) / D ** 0.5
    mask = torch.arange(P).view(1, -1) > torch.arange(P - last, P).view(-1, 1)
    sc = sc.masked_fill(mask, float("-inf"))
    ref = torch.softmax(sc, dim=-1) @ vv
    assert rel_l2(out.cpu().numpy(), ref.numpy()) < 1e-5
    # the pool holds every position's K and V in every layer of its block
    got_k = torch.stack([pool[bt[p // B], :, 0, :, p % B, :] for p in range(P)], dim=0).cpu()
    assert rel_l2(got_k[:, 0].transpose(0, 1).numpy(), k.numpy()) < 1e-5
    assert torch.equal(got_k[:, 0], got_k[:, 1])
    got_v = torch.stack([pool[bt[p // B], 1, 1, :, p % B, :] for p in range(P)], dim=1).cpu()
    assert rel_l2(got_v.numpy(), v.numpy()) < 1e-5


@pytest.mark.parametrize("m,H,V,norm", [(17, 4096, 128256, True), (64, 4096, 128256, False),
                                        (65, 896, 1000, True), (130, 256, 130, False),
                                        (20, 896, 151936, True), (1, 512, 777, False)])
def test_lm_head_tensor_core_split_weight(m, H, V, norm):
    """ksh_lm_head_argmax_tc on the split fp16 weight: logits within 1e-5 of
    the largest |logit| of a float64 reference (the other lm_head paths'
    bound), tokens the first index of the maximum of those logits (a tie
    between duplicate weight rows goes to the lower index), more than 64 rows
    in several launches, a workspace that starts as 0xFF bytes and no write
    past the size the query asked for."""
    from kshipra_b200 import _lib
    gen = torch.Generator().manual_seed(m * 13 + H + V)
    w = torch.randn((V, H), generator=gen) * 0.02
    w[V // 3] = w[V - 5]
    x = torch.randn((m, H), generator=gen)
    x[0] = w[V - 5] * 50
    nw = 1.0 + 0.1 * torch.randn(H, generator=gen)
    wc, xc, nc = w.cuda(), x.cuda(), nw.cuda()
    hi = torch.empty((V, H), dtype=torch.float16, device="cuda")
    lo = torch.empty_like(hi)
    inv = torch.empty(V, device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.call("ksh_lm_head_split_weight", wc.data_ptr(), V, H, hi.data_ptr(), lo.data_ptr(),
              inv.data_ptr(), flags.data_ptr(), _lib.stream_ptr())
    # the split reconstructs the weight to about 2^-22 of each row's maximum
    rec = (hi.double() + lo.double()) * inv.double().view(-1, 1)
    err = (rec.cpu() - w.double()).abs().max(dim=1).values / w.double().abs().max(dim=1).values
    assert float(err.max()) < 2.0 ** -21 and int(flags.item()) == 0
    need = int(_lib.lib().ksh_lm_head_tc_workspace_size(m, H, V))
    guard = 1 << 16
    ws = torch.full((need + guard,), 0xFF, dtype=torch.uint8, device="cuda")
    ws[need:] = 0xAB
    logits = torch.empty((m, V), device="cuda")
    tok = torch.full((m,), -7, dtype=torch.int64, device="cuda")
    xd = x.double()
    if norm:
        xd = xd * torch.rsqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.double()
    ref = xd @ w.double().T
    for _ in range(2):
        _lib.call("ksh_lm_head_argmax_tc", xc.data_ptr(), m, H, nc.data_ptr() if norm else None,
                  1e-6, hi.data_ptr(), lo.data_ptr(), inv.data_ptr(), V, logits.data_ptr(),
                  tok.data_ptr(), ws.data_ptr(), need, _lib.stream_ptr())
        torch.cuda.synchronize()
        assert bool((ws[need:] == 0xAB).all())
        lg = logits.cpu()
        assert float((lg.double() - ref).abs().max()) <= 1e-5 * float(ref.abs().max())
        assert tok.cpu().tolist() == torch.argmax(lg, dim=1).tolist()
        assert int(tok[0]) == V // 3
    # argmax only (no logits buffer) gives the same tokens
    tok2 = torch.full((m,), -7, dtype=torch.int64, device="cuda")
    _lib.call("ksh_lm_head_argmax_tc", xc.data_ptr(), m, H, nc.data_ptr() if norm else None, 1e-6,
              hi.data_ptr(), lo.data_ptr(), inv.data_ptr(), V, None, tok2.data_ptr(),
              ws.data_ptr(), need, _lib.stream_ptr())
    torch.cuda.synchronize()
    assert tok2.cpu().tolist() == tok.cpu().tolist()


def test_model_lm_head_paths_agree():
    """The model's lm_head above 16 rows (tensor cores, split weight) and the
    fp32 GEMV path give the same tokens and logits within 1e-5."""
    from kshipra_b200.config import TINY_LLAMA
    from kshipra_b200.model import KshipraModel
    from kshipra_b200.weights import synthetic_state_dict
    km = KshipraModel(config=TINY_LLAMA, state_dict=synthetic_state_dict(TINY_LLAMA, seed=0),
                      quantize="int8")
    x = torch.randn((40, TINY_LLAMA.hidden), generator=torch.Generator().manual_seed(5)).cuda()
    lg_tc = torch.empty((40, TINY_LLAMA.vocab), device="cuda")
    tok_tc = torch.empty(40, dtype=torch.int64, device="cuda")
    km._lm_head_argmax(x, tok_tc, logits=lg_tc)
    km.lm_tc = False
    lg_f = torch.empty_like(lg_tc)
    tok_f = torch.empty_like(tok_tc)
    km._lm_head_argmax(x, tok_f, logits=lg_f)
    scale = float(lg_f.abs().max())
    assert float((lg_tc - lg_f).abs().max()) <= 1e-5 * scale
    # the same token wherever the fp32 top-2 margin exceeds the logits' tolerance
    top2 = lg_f.topk(2, dim=1).values
    clear = (top2[:, 0] - top2[:, 1]) > 2e-5 * scale
    assert bool(clear.any())
    assert tok_tc[clear].tolist() == tok_f[clear].tolist()
    lg_at = lg_f.gather(1, tok_tc.view(-1, 1)).view(-1)
    assert bool(((top2[:, 0] - lg_at) <= 2e-5 * scale).all())


@pytest.mark.parametrize("scheme", ["int4", "int8"])
@pytest.mark.parametrize("m", [1, 8, 40, 130])
def test_linear_with_outlier_features(scheme, m):
    """Activation rows with a few outlier features, 1e3 to 1e4 times the rest
    of their row (as real checkpoints have), through every quantized-linear
    path: one row (INT4 dp4a GEMV / INT8 tensor-core GEMV), 8 rows (tensor-core
    decode kernel), 40 rows (batched-decode kernel), 130 rows (prefill GEMM).
    The activations are carried as 22-bit fixed point per 32-element vector
    (dp4a) or per row (hi + lo fp16), so the features next to an outlier keep
    fewer bits; the bound is the one the other linear tests use, per row
    against float64 with the dequantized weight: max |error| <= 2e-5 x
    max |y|, with the fp32 reference's own error printed beside it."""
    from kshipra_b200.quantization import (linear_launch, quantize_int4_per_group,
                                           quantize_int8_per_channel)
    gen = torch.Generator().manual_seed(77 + m)
    K, N = 4096, 512
    x = torch.randn((m, K), generator=gen)
    for r in range(m):
        idx = torch.randint(0, K, (4,), generator=gen)
        x[r, idx] *= torch.tensor([1e3, -3e3, 6e3, 1e4])
    w = torch.randn((N, K), generator=gen) * 0.03
    if scheme == "int8":
        qw = quantize_int8_per_channel(w.cuda())
        wd = oq.dequantize_int8(*oq.quantize_int8_per_channel(w.numpy()))
    else:
        qw = quantize_int4_per_group(w.cuda(), 128)
        p, s, _ = oq.quantize_int4_per_group(w.numpy(), 128)
        wd = oq.dequantize_int4(p, s, K, 128)
    y64 = x.double().numpy() @ wd.astype(np.float64).T
    y32 = (x @ torch.from_numpy(wd.astype(np.float32)).T).double().numpy()   # fp32 F.linear
    y = torch.empty((m, N), device="cuda")
    linear_launch(x.cuda(), qw, None, None, y)
    den = np.abs(y64).max(axis=1)
    err = np.abs(y.cpu().numpy() - y64).max(axis=1) / den
    err32 = np.abs(y32 - y64).max(axis=1) / den
    assert err.max() <= 2e-5, (scheme, m, float(err.max()), float(err32.max()))


@pytest.mark.parametrize("scheme,g", [("int8", 0), ("int4", 128), ("int4", 64)])
@pytest.mark.parametrize("m,k,n", [(600, 1000, 640), (2048, 4096, 768), (512, 896, 1216)])
def test_prefill_gemm_widened_weight_path_matches(scheme, g, m, k, n):
    """The prefill GEMM with the weight widened to fp16 once per call (PRE)
    and with per-tile widening give the same output, bit for bit (the same
    MMAs in the same order), for the store and SwiGLU epilogues, with bias
    and residual, and K not a multiple of the 128-wide group."""
    from kshipra_b200 import _lib
    from kshipra_b200.quantization import (linear_launch, quantize_int4_per_group,
                                           quantize_int8_per_channel, swiglu_launch)
    gen = torch.Generator().manual_seed(m + k + n + g)
    x = torch.randn((m, k), generator=gen).cuda()
    w = (torch.randn((n, k), generator=gen) * 0.02).cuda()
    b = torch.randn((n,), generator=gen).cuda()
    res = torch.randn((m, n), generator=gen).cuda()
    qw = quantize_int8_per_channel(w) if scheme == "int8" else quantize_int4_per_group(w, g)
    outs = []
    prev = _lib.lib().ksh_set_gemm_predeq(512)
    try:
        for mode in (512, 0):
            _lib.lib().ksh_set_gemm_predeq(mode)
            y = res.clone()
            linear_launch(x, qw, None, b, y, residual=y)
            h = torch.empty((m, n // 2), device="cuda")
            swiglu_launch(x, qw, None, n // 2, h)
            torch.cuda.synchronize()
            outs.append((y.cpu(), h.cpu()))
    finally:
        _lib.lib().ksh_set_gemm_predeq(prev)
    assert torch.equal(outs[0][0], outs[1][0])
    assert torch.equal(outs[0][1], outs[1][1])
