"""tcgen05 int8 GEMM + fused epilogues vs the CPU oracle (gemm_int8_fused, src/gemm.rs:630-671, and
the row kernels of src/simd_math.rs). int32 accumulators and every fp32 / int8 output are compared
bit for bit, except the GELU epilogue, whose reciprocal differs from the reference's rcp_ps estimate
by about one ulp (see test_gelu_quant_epilogue)."""
import numpy as np
import pytest
import torch

from conftest import rng
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_case(M, K, N, seed):
    r = rng(seed)
    a = r.integers(-127, 128, size=(M, K), dtype=np.int8)
    w = np.clip(np.rint(r.normal(0, 40, size=(N, K))), -127, 127).astype(np.int8)
    a_s = r.uniform(1e-3, 1e-2, M).astype(np.float32)
    w_s = r.uniform(1e-3, 1e-2, N).astype(np.float32)
    b = r.normal(0, 0.02, N).astype(np.float32)
    return a, w, a_s, w_s, b


@pytest.mark.parametrize("K,N", [(384, 1152), (384, 768), (384, 384), (1536, 384)])
@pytest.mark.parametrize("M", [1, 37, 128, 300])
def test_f32_epilogue_bit_exact(engine, M, K, N):
    a, w, a_s, w_s, b = make_case(M, K, N, M * 7 + N)
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    acc = torch.zeros(M, N, dtype=torch.int32, device="cuda")
    engine.gemm_i8(0, dev(a), dev(a_s), dev(w), dev(w_s), dev(b), out=out, acc=acc)
    engine.sync()
    ref_out, ref_acc = orc.gemm(orc.BACKEND_AVX2 if orc.lib().or_has_avx2_fma() else orc.BACKEND_SCALAR, a, a_s, w, w_s, b)
    np.testing.assert_array_equal(acc.cpu().numpy(), a.astype(np.int64) @ w.astype(np.int64).T)
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    np.testing.assert_array_equal(out.cpu().numpy(), ref_out)


# ae_gemm_i8 takes the LayerNorm epilogues fused into the GEMM from 74 row tiles (9,345+ rows) and
# as a plain GEMM + row kernel below: both sides of the switch are checked
@pytest.mark.parametrize("K", [384, 1536])
@pytest.mark.parametrize("M", [1, 100, 256, 333, 9473])
def test_ln_quant_epilogue_bit_exact(engine, M, K):
    N = 384
    a, w, a_s, w_s, b = make_case(M, K, N, 11 * M + K)
    r = rng(M + K)
    res = r.normal(0, 1, (M, N)).astype(np.float32)
    g = (1 + r.normal(0, 0.05, N)).astype(np.float32)
    be = r.normal(0, 0.02, N).astype(np.float32)
    inv_s = r.uniform(0.5, 2.0, N).astype(np.float32)
    d_res = dev(res)
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    q = torch.zeros(M, N, dtype=torch.int8, device="cuda")
    sc = torch.zeros(M, dtype=torch.float32, device="cuda")
    engine.gemm_i8(1, dev(a), dev(a_s), dev(w), dev(w_s), dev(b), res=d_res, gamma=dev(g), beta=dev(be),
                   inv_smooth=dev(inv_s), out=out, out_q=q, out_scale=sc)
    engine.sync()
    h, _ = orc.gemm(orc.BACKEND_SCALAR, a, a_s, w, w_s, b, res)
    y, q_ref, s_ref = orc.ln_quant_rows(h, g, be, inv_s)
    np.testing.assert_array_equal(out.cpu().numpy(), y)
    np.testing.assert_array_equal(q.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(sc.cpu().numpy(), s_ref)


@pytest.mark.parametrize("M", [200, 9600])
def test_ln_quant_in_place(engine, M):
    """The forward pass writes the LayerNorm output over the residual it reads."""
    K, N = 384, 384
    a, w, a_s, w_s, b = make_case(M, K, N, 5)
    r = rng(9)
    res = r.normal(0, 1, (M, N)).astype(np.float32)
    g = (1 + r.normal(0, 0.05, N)).astype(np.float32)
    be = r.normal(0, 0.02, N).astype(np.float32)
    inv_s = r.uniform(0.5, 2.0, N).astype(np.float32)
    d_res = dev(res)
    d_a = dev(a)
    d_as = dev(a_s)
    engine.gemm_i8(1, d_a, d_as, dev(w), dev(w_s), dev(b), res=d_res, gamma=dev(g), beta=dev(be),
                   inv_smooth=dev(inv_s), out=d_res, out_q=d_a, out_scale=d_as)
    engine.sync()
    h, _ = orc.gemm(orc.BACKEND_SCALAR, a, a_s, w, w_s, b, res)
    y, q_ref, s_ref = orc.ln_quant_rows(h, g, be, inv_s)
    np.testing.assert_array_equal(d_res.cpu().numpy(), y)
    np.testing.assert_array_equal(d_a.cpu().numpy(), q_ref)
    np.testing.assert_array_equal(d_as.cpu().numpy(), s_ref)


@pytest.mark.parametrize("M", [1, 77, 128, 390, 2000])
def test_gelu_quant_epilogue(engine, M):
    """GELU + SmoothQuant + row quantization (gelu_smooth_quantize_row_avx2). The GPU restates the
    reference's rational GELU with a correctly rounded reciprocal where the reference uses the
    12-bit rcp_ps estimate, so the two agree to about one ulp: int8 outputs may differ by one
    level at a rounding boundary (rarely), the row scales by at most a few ulp. Up to 12 row
    tiles the 1,536 columns are 12 slices of 128 (a 12-CTA cluster), beyond that 6 of 256."""
    K, N = 384, 1536
    a, w, a_s, w_s, b = make_case(M, K, N, 3 * M)
    inv_s = rng(M).uniform(0.5, 2.0, N).astype(np.float32)
    q = torch.zeros(M, N, dtype=torch.int8, device="cuda")
    sc = torch.zeros(M, dtype=torch.float32, device="cuda")
    acc = torch.zeros(M, N, dtype=torch.int32, device="cuda")
    engine.gemm_i8(2, dev(a), dev(a_s), dev(w), dev(w_s), dev(b), inv_smooth=dev(inv_s), out_q=q, out_scale=sc, acc=acc)
    engine.sync()
    h, ref_acc = orc.gemm(orc.BACKEND_SCALAR, a, a_s, w, w_s, b)
    np.testing.assert_array_equal(acc.cpu().numpy(), ref_acc)
    _, q_ref, s_ref = orc.gelu_quant_rows(h, inv_s)
    np.testing.assert_allclose(sc.cpu().numpy(), s_ref, rtol=5e-7)
    dq = np.abs(q.cpu().numpy().astype(np.int32) - q_ref.astype(np.int32))
    assert dq.max() <= 1
    assert (dq > 0).mean() < 1e-4


@pytest.mark.parametrize("M", [1, 64, 129, 9473])
def test_final_ln_l2_epilogue_bit_exact(engine, M):
    K, N = 1536, 384
    a, w, a_s, w_s, b = make_case(M, K, N, 13 + M)
    r = rng(M)
    res = r.normal(0, 1, (M, N)).astype(np.float32)
    g = (1 + r.normal(0, 0.05, N)).astype(np.float32)
    be = r.normal(0, 0.02, N).astype(np.float32)
    out = torch.zeros(M, N, dtype=torch.float32, device="cuda")
    engine.gemm_i8(3, dev(a), dev(a_s), dev(w), dev(w_s), dev(b), res=dev(res), gamma=dev(g), beta=dev(be), out=out)
    engine.sync()
    h, _ = orc.gemm(orc.BACKEND_SCALAR, a, a_s, w, w_s, b, res)
    ref = np.empty_like(h)
    for i in range(M):
        row = np.ascontiguousarray(h[i])
        orc.lib().or_layernorm_inplace_row(orc._p(row, orc.C.c_float), orc._p(g, orc.C.c_float), orc._p(be, orc.C.c_float), N)
        orc.lib().or_l2_normalize(orc._p(row, orc.C.c_float), N)
        ref[i] = row
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
