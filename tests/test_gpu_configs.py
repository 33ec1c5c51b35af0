"""The benchmark configurations themselves pass the parity bar, at their full
sizes where the checker can follow:

  config 5  int8 GEMMs at (K, N) = (384, 1152), (384, 384), (384, 1536), (1536, 384) and
            M = 512, 8192, 65536: int32 accumulators equal to an independent exact int8 matmul on
            the GPU (torch._int_mm); the fp32 epilogue equal to fma(float(acc), a_s * w_s, bias)
            evaluated in float64 and rounded once (double rounding can move a result by one ulp,
            so one ulp is allowed); and 64 x 12 x 512 x 32 attention (whose exact order the
            oracle checks at smaller sizes) agreeing with a float64 softmax attention
  config 3  the whole 512 x 128-token batch against the oracle (cos >= 0.9999, max-abs <= 2e-3)
  config 4  sequences drawn from the log-uniform [8, 512] length distribution, ragged-packed,
            against the oracle
"""
import os

import numpy as np
import pytest
import torch

from conftest import COS_MIN, MAXABS_MAX, rng
from arctic_embed_s_int8 import synth

pytestmark = pytest.mark.gpu


def close_rows(got, ref):
    cos = np.sum(got * ref, 1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))
    return float(cos.min()), float(np.abs(got - ref).max())


@pytest.mark.parametrize("K,N", [(384, 1152), (384, 384), (384, 1536), (1536, 384)])
@pytest.mark.parametrize("M", [512, 8192, 65536])
def test_config5_gemm_full_size(engine, M, K, N):
    g = torch.Generator(device="cuda").manual_seed(M + K + N)
    a = torch.randint(-127, 128, (M, K), device="cuda", generator=g, dtype=torch.int8)
    w = torch.clamp(torch.round(torch.randn(N, K, device="cuda", generator=g) * 40), -127, 127).to(torch.int8)
    a_s = torch.rand(M, device="cuda", generator=g) * 9e-3 + 1e-3
    w_s = torch.rand(N, device="cuda", generator=g) * 9e-3 + 1e-3
    b = torch.randn(N, device="cuda", generator=g) * 0.02
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    acc = torch.empty(M, N, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()  # the engine runs on its own stream: the inputs must be complete
    engine.gemm_i8(0, a, a_s, w, w_s, b, out=out, acc=acc)
    engine.sync()
    ref_acc = torch._int_mm(a, w.t().contiguous())
    assert torch.equal(acc, ref_acc)
    ref = (acc.to(torch.float32).double() * (a_s[:, None] * w_s[None, :]).double() + b[None, :].double()).float()
    ulp = torch.abs(ref.view(torch.int32) - out.view(torch.int32))
    assert int(ulp.max()) <= 1 and float((ulp > 0).float().mean()) < 1e-4


def test_config5_attention(engine):
    n, L = 64, 512
    g = torch.Generator(device="cuda").manual_seed(5)
    qkv = torch.randn(n * L, 1152, device="cuda", generator=g)
    cu = torch.arange(0, n * L + 1, L, device="cuda", dtype=torch.int32)
    ctx = torch.empty(n * L, 384, device="cuda")
    torch.cuda.synchronize()  # the engine runs on its own stream: the inputs must be complete
    engine.attention_f32(qkv, cu, n, L, ctx)
    engine.sync()
    x = qkv.double().view(n, L, 3, 12, 32)
    q, k, v = x[:, :, 0].transpose(1, 2), x[:, :, 1].transpose(1, 2), x[:, :, 2].transpose(1, 2)
    p = torch.softmax((q / np.sqrt(32.0)) @ k.transpose(-1, -2), dim=-1)
    ref = (p @ v).transpose(1, 2).reshape(n * L, 384)
    assert float((ctx.double() - ref).abs().max()) < 2e-5


def test_config3_full_batch(engine, oracle_model):
    r = rng(303)
    seqs = [synth.token_ids(128, r) for _ in range(512)]
    got = engine.forward_ragged(seqs)
    ref = oracle_model.embed_batch(seqs, os.cpu_count() or 1)
    cos, mx = close_rows(got, ref)
    assert cos >= COS_MIN and mx <= MAXABS_MAX, (cos, mx)


def test_config4_ragged_sample(engine, oracle_model):
    r = rng(404)
    lens = np.exp(r.uniform(np.log(8), np.log(512), 256)).astype(int)
    seqs = [synth.token_ids(int(L), r) for L in lens]
    got = engine.forward_ragged(seqs)
    ref = oracle_model.embed_batch(seqs, os.cpu_count() or 1)
    cos, mx = close_rows(got, ref)
    assert cos >= COS_MIN and mx <= MAXABS_MAX, (cos, mx)
