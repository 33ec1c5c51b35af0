"""The int8 attention mode (the reference's SME scheme, attention_heads_sme,
src/simd_math.rs:1933-2186) on the B200 vs the oracle's restatement of it: bit for bit where a
sequence has no keys past its last complete 8-key block (the only admitted difference is exp2 of
those last keys: CUDA's exp2f vs glibc's), and the full forward in the int8 mode within the
north-star tolerance of the oracle's int8 mode."""
import numpy as np
import pytest
import torch

from conftest import COS_MIN, MAXABS_MAX, rng
from arctic_embed_s_int8 import ATTENTION_EXACT, ATTENTION_INT8, Engine, synth
from oracle import oracle as orc
from test_oracle import bench_qkv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def engine8(pack_path):
    eng = Engine(0).load_file(pack_path).set_attention_mode(ATTENTION_INT8)
    yield eng
    eng.close()


@pytest.fixture(scope="module")
def oracle8(pack_path):
    return orc.OracleModel(pack_path).set_attention_mode(orc.ATTENTION_INT8)


def run_i8(engine, qkv, lens):
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    ctx = torch.full((qkv.shape[0], 384), float("nan"), dtype=torch.float32, device="cuda")
    engine.attention_i8(torch.from_numpy(qkv).cuda(), torch.from_numpy(cu.astype(np.int32)).cuda(), len(lens),
                        max(lens), ctx)
    engine.sync()
    return ctx.cpu().numpy(), cu


@pytest.mark.parametrize("lens", [[1, 2, 7], [8, 15, 16, 17], [64, 33, 100], [128] * 6, [512, 257], [512] * 3])
def test_attention_i8_matches_oracle(engine8, lens):
    r = rng(900 + sum(lens))
    T = sum(lens)
    qkv = r.normal(0, 1, (T, 1152)).astype(np.float32)
    qkv[:lens[0]] = bench_qkv(lens[0])  # the reference benchmark's input for the first sequence
    got, cu = run_i8(engine8, qkv, lens)
    for s, L in enumerate(lens):
        b, e = int(cu[s]), int(cu[s + 1])
        ref = orc.attention_i8(qkv[b:e])
        if L % 8 == 0:
            np.testing.assert_array_equal(got[b:e], ref, err_msg=f"L={L}")
        else:
            assert (got[b:e] == ref).mean() > 0.99, L
            np.testing.assert_allclose(got[b:e], ref, rtol=0, atol=1e-3 * float(np.abs(ref).max()))


@pytest.mark.parametrize("L", [8, 15, 16, 24, 100, 128, 512])
def test_int8_mode_forward_matches_oracle(engine8, oracle8, L):
    ids = synth.token_ids(L, rng(3000 + L))
    got = engine8.forward_cls(ids)
    ref = oracle8.forward_cls(ids)
    cos = float(np.dot(got, ref) / (np.linalg.norm(got) * np.linalg.norm(ref)))
    assert cos >= COS_MIN and float(np.abs(got - ref).max()) <= MAXABS_MAX, (L, cos)


def test_int8_mode_batches_and_switching(engine8, oracle8, engine):
    """Packed batches (with sequences under the 16-token crossover mixed in, and through the
    device-pointer entry) give each sequence's single-sequence result; sequences under 16 tokens
    equal the fp32 mode; switching the mode back restores the fp32 results."""
    r = rng(31)
    lens = [3, 20, 15, 128, 16, 300, 9, 64, 512, 31]
    seqs = [synth.token_ids(L, r) for L in lens]
    got = engine8.forward_ragged(seqs)
    single = np.stack([engine8.forward_cls(s) for s in seqs])
    np.testing.assert_array_equal(got, single)
    for s, g in zip(seqs, got):
        ref = oracle8.forward_cls(s)
        cos = float(np.dot(g, ref) / (np.linalg.norm(g) * np.linalg.norm(ref)))
        assert cos >= COS_MIN and float(np.abs(g - ref).max()) <= MAXABS_MAX, (len(s), cos)
    from arctic_embed_s_int8 import pack_sequences

    ids, cu = pack_sequences(seqs)
    out = torch.zeros(len(seqs), 384, dtype=torch.float32, device="cuda")
    engine8.forward_device(torch.from_numpy(ids.view(np.int16)).cuda(), torch.from_numpy(cu.view(np.int32)).cuda(),
                           len(seqs), int(cu[-1]), 512, out)
    engine8.sync()
    np.testing.assert_array_equal(out.cpu().numpy(), got)
    exact = np.stack([engine.forward_cls(s) for s in seqs])
    for L, g, x in zip(lens, got, exact):
        assert np.array_equal(g, x) == (L < 16), L
    assert engine8.attention_mode == ATTENTION_INT8
    engine8.set_attention_mode(ATTENTION_EXACT)
    try:
        np.testing.assert_array_equal(engine8.forward_cls(seqs[3]), exact[3])
    finally:
        engine8.set_attention_mode(ATTENTION_INT8)
