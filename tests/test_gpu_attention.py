"""Segment-masked fp32 attention vs the oracle's per-(head, query) attention
(compute_scores_head32 + softmax_inplace + weighted_sum_head32, src/simd_math.rs:2953-3070), on
the layout of the fused QKV buffer (src/model.rs:294-321)."""
import numpy as np
import pytest
import torch

from conftest import rng
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def ref_attention(qkv, cu):
    out = np.zeros((qkv.shape[0], 384), np.float32)
    for s in range(len(cu) - 1):
        b, e = int(cu[s]), int(cu[s + 1])
        for h in range(12):
            k = np.ascontiguousarray(qkv[b:e, 384 + 32 * h: 384 + 32 * h + 32])
            v = np.ascontiguousarray(qkv[b:e, 768 + 32 * h: 768 + 32 * h + 32])
            for t in range(b, e):
                out[t, 32 * h: 32 * h + 32] = orc.attention_query(qkv[t, 32 * h: 32 * h + 32], k, v)
    return out


@pytest.mark.parametrize("lens", [[1], [2, 3, 5], [8, 15, 16, 17], [31, 33, 64], [100, 1, 7], [128], [257], [512]])
def test_attention_matches_oracle(engine, lens):
    r = rng(sum(lens))
    T = sum(lens)
    qkv = r.normal(0, 1, (T, 1152)).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    ctx = torch.zeros(T, 384, dtype=torch.float32, device="cuda")
    engine.attention_f32(torch.from_numpy(qkv).cuda(), torch.from_numpy(cu.astype(np.int32)).cuda(), len(lens),
                         max(lens), ctx)
    engine.sync()
    got = ctx.cpu().numpy()
    ref = ref_attention(qkv, cu)
    # identical operation order; the only admitted difference is the scalar exp of softmax tail
    # elements (libm expf on the CPU, a correctly rounded exp on the GPU): at most a few ulp
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6)
    assert (got == ref).mean() > 0.99


def test_attention_two_queries_per_thread_matches_oracle(engine):
    """25 sequences of 65..128 keys (300 (sequence, head) pairs) take the kernel whose threads hold
    two queries each, with K / V staged dim-major; odd lengths and partial 16-key chunks included."""
    r = rng(65)
    lens = [128, 65, 127, 97, 100] + list(r.integers(65, 129, 20))
    T = sum(lens)
    qkv = r.normal(0, 1, (T, 1152)).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    ctx = torch.zeros(T, 384, dtype=torch.float32, device="cuda")
    engine.attention_f32(torch.from_numpy(qkv).cuda(), torch.from_numpy(cu.astype(np.int32)).cuda(), len(lens),
                         max(lens), ctx)
    engine.sync()
    got = ctx.cpu().numpy()
    ref = ref_attention(qkv, cu)
    np.testing.assert_allclose(got, ref, rtol=0, atol=2e-6)
    assert (got == ref).mean() > 0.99


@pytest.mark.parametrize("lens", [[128] * 25, [128], [512], [64] * 30, [144] * 3])
def test_attention_bit_exact_without_scalar_tail(engine, lens):
    """Lengths that are multiples of 16 have no softmax tail element (every exponential is the
    reference's 8-wide Cody-Waite polynomial, computed on the packed f32x2 pipe): the attention then
    equals the oracle bit for bit, whichever kernel takes the batch (two queries per thread for
    25 x 128, the single-sequence dim-major kernels at 128 and 512, the key-pair kernel for 30 x 64,
    the few-sequence kernel for 3 x 144)."""
    r = rng(sum(lens) + 1)
    T = sum(lens)
    qkv = r.normal(0, 1, (T, 1152)).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    ctx = torch.zeros(T, 384, dtype=torch.float32, device="cuda")
    engine.attention_f32(torch.from_numpy(qkv).cuda(), torch.from_numpy(cu.astype(np.int32)).cuda(), len(lens),
                         max(lens), ctx)
    engine.sync()
    np.testing.assert_array_equal(ctx.cpu().numpy(), ref_attention(qkv, cu))
