"""The CPU oracle (C++ restatement of the reference's x86 path), checked without a GPU.

The reference's golden vectors (tests/data/*.json of the reference crate) are tied to the real
model weights, which are not available, so the oracle is pinned by (1) an independent float64
NumPy forward of the same synthetic model, with the reference's own accuracy thresholds against
its FP32 model (tests/accuracy_test.rs:109-132), (2) the reference's invariants (every SIMD
backend vs scalar, ragged vs single, pruned layer 11: tests/accuracy_test.rs:134-207), and
(3) committed golden fixtures of this synthetic pack (tests/golden/)."""
import os

import numpy as np
import pytest

from conftest import rng
from arctic_embed_s_int8 import ae8, synth
from oracle import oracle as orc

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "synthetic_seed0.npz")


@pytest.fixture(scope="module")
def fp32_model():
    return synth.make_fp32_model(0)


def test_accuracy_vs_float64_forward(oracle_model, fp32_model):
    """tests/accuracy_test.rs:109-132: cos > 0.9985 per record, mean > 0.9992 (vs the FP model)."""
    coss = []
    for i, L in enumerate([8, 17, 33, 64, 128, 200]):
        ids = synth.token_ids(L, rng(100 + i))
        e = oracle_model.forward_cls(ids)
        ref = synth.fp_forward(fp32_model, ids)
        coss.append(float(e @ ref))
        assert abs(np.linalg.norm(e) - 1.0) < 1e-5
    assert min(coss) > 0.9985 and np.mean(coss) > 0.9992, coss


def test_backends_match(pack_path):
    """tests/accuracy_test.rs:154-207: every supported backend vs Scalar, cos > 0.999. The int32
    accumulators are exact in every backend, so AVX-VNNI and AVX2 agree bit for bit."""
    ids = synth.token_ids(40, rng(1))
    sc = orc.OracleModel(pack_path, orc.BACKEND_SCALAR).forward_cls(ids)
    outs = {}
    for b in (orc.BACKEND_AVX_VNNI, orc.BACKEND_AVX2):
        try:
            outs[b] = orc.OracleModel(pack_path, b).forward_cls(ids)
        except ValueError:
            continue  # backend not supported by this CPU
        assert float(outs[b] @ sc) > 0.999
    if len(outs) == 2:
        np.testing.assert_array_equal(outs[orc.BACKEND_AVX_VNNI], outs[orc.BACKEND_AVX2])


def test_ragged_equals_single(oracle_model):
    """tests/accuracy_test.rs:134-150 (cos > 0.99999); on x86 the packed path is bit-identical."""
    seqs = [synth.token_ids(L, rng(L)) for L in [5, 9, 3, 12, 1, 7]]
    got = oracle_model.forward_ragged(seqs)
    for s, g in zip(seqs, got):
        np.testing.assert_array_equal(g, oracle_model.forward_cls(s))


def test_embed_batch_threads_and_order(oracle_model):
    """embed_batch (src/lib.rs:138-260): results by index, independent of the thread count."""
    r = rng(3)
    seqs = [synth.token_ids(int(L), r) for L in r.integers(2, 40, 24)]
    a = oracle_model.embed_batch(seqs, 1)
    b = oracle_model.embed_batch(seqs, 4)
    np.testing.assert_array_equal(a, b)
    for s, e in zip(seqs[:6], a[:6]):
        np.testing.assert_array_equal(e, oracle_model.forward_cls(s))


def test_pruned_layer11_layout(quantized):
    """tests/accuracy_test.rs:203-207: layer 11's fused qkv is pruned (no weights); q_only/kv_only
    carry the same input smoothing as the fused QKV would."""
    l11 = quantized.layers[11]
    assert l11.qkv.n_out == 0 and l11.qkv.w_q.size == 0 and l11.qkv.inv_smooth.size == 384
    assert l11.q_only.w_q.shape == (384, 384) and l11.kv_only.w_q.shape == (768, 384)
    np.testing.assert_array_equal(l11.q_only.inv_smooth, l11.qkv.inv_smooth)
    for l in range(11):
        assert quantized.layers[l].q_only is None and quantized.layers[l].qkv.w_q.shape == (1152, 384)


def test_truncation(oracle_model):
    ids = synth.token_ids(600, rng(4))
    np.testing.assert_array_equal(oracle_model.forward_cls(ids), oracle_model.forward_cls(ids[:512]))


def test_golden_fixture(pack_path, oracle_model):
    """Committed fixture: the seeded pack's digest and the oracle's embeddings of a few sequences,
    with the fp32 attention and in the int8 attention mode."""
    g = np.load(GOLDEN)
    assert synth.file_sha256(pack_path) == str(g["pack_sha256"])
    m8 = orc.OracleModel(pack_path).set_attention_mode(orc.ATTENTION_INT8)
    for i in range(int(g["n"])):
        ids = g[f"ids_{i}"]
        np.testing.assert_allclose(oracle_model.forward_cls(ids), g[f"emb_{i}"], rtol=0, atol=1e-6)
        np.testing.assert_allclose(m8.forward_cls(ids), g[f"emb_i8_{i}"], rtol=0, atol=1e-6)


def test_pack_round_trip_and_errors(pack_path, tmp_path):
    m = ae8.read_ae8(pack_path)
    p = tmp_path / "copy.ae8"
    ae8.write_ae8(m, p)
    assert open(p, "rb").read() == open(pack_path, "rb").read()
    raw = open(pack_path, "rb").read()
    with pytest.raises(ae8.Ae8FormatError, match="magic"):
        ae8.read_ae8(b"XXXXXXXX" + raw[8:])
    with pytest.raises(ae8.Ae8FormatError):
        ae8.read_ae8(raw[: len(raw) // 2])
    with pytest.raises(ValueError, match="magic"):
        orc.OracleModel.from_bytes(b"XXXXXXXX" + raw[8:])
    with pytest.raises(ValueError, match="truncated"):
        orc.OracleModel.from_bytes(raw[: len(raw) - 100])


def test_row_kernels_known_answers():
    """Row kernels of src/simd_math.rs on hand-checkable inputs."""
    x = np.zeros(384, np.float32)
    x[5] = 2.0
    s = np.ones(384, np.float32)
    q, sc = orc.smooth_quant_rows(x[None], s)
    assert sc[0] == np.float32(2.0) / np.float32(127.0) and q[0, 5] == 127 and np.count_nonzero(q) == 1
    z = np.zeros((1, 384), np.float32)  # all-zero row: max_abs floor 1e-8, q = 0
    q, sc = orc.smooth_quant_rows(z, s)
    assert sc[0] == np.float32(1e-8) / np.float32(127.0) and not q.any()
    y = orc.gelu_ref(np.array([0.0, 10.0, -10.0, 1.0], np.float32))
    assert y[0] == 0.0 and y[1] == 10.0 and y[2] == 0.0 and abs(y[3] - 0.8413447) < 1e-5


# ------------------------------------------------------------------------------------ int8 attention
def bench_qkv(L):
    """The reference's attention micro-benchmark input (examples/attn_bench.rs:19-21):
    qkv[i] = ((i * 2654435761) % 1000) / 300 - 1.6, as f32 [L, 1152]."""
    i = np.arange(L * 1152, dtype=np.uint64)
    v = ((i * np.uint64(2654435761)) % np.uint64(1000)).astype(np.float32) / np.float32(300.0) - np.float32(1.6)
    return v.reshape(L, 1152)


def np_attention_i8(qkv):
    """Independent NumPy statement of the reference's int8 attention scheme (attention_heads_sme,
    src/simd_math.rs:1933-2186) for one sequence: float32 elementwise steps, exact integer sums,
    the polynomial's fused multiply-adds as float64 products and sums (exact products; a double
    rounding only at an exact float32 midpoint)."""
    f32 = np.float32
    L = qkv.shape[0]
    out = np.zeros((L, 384), f32)
    k_mul = (f32(1.0) / np.sqrt(f32(32.0))) * f32(1.4426950408889634)

    def quant_rows(x, mul):
        m = np.maximum(np.abs(x).max(axis=1), f32(1e-8))
        q = np.clip(np.rint(x * (f32(127.0) / m)[:, None]), -128, 127).astype(np.int64)
        return q, (m / f32(127.0)) * f32(mul)

    c = [f32(f32(0.999857) * f32(16383.0)), f32(f32(0.6963853) * f32(16383.0)),
         f32(f32(0.22511937) * f32(16383.0)), f32(f32(0.07842169) * f32(16383.0))]

    def fma(a, b, d):
        return (a.astype(np.float64) * b.astype(np.float64) + np.float64(d)).astype(f32)

    L8 = L - L % 8
    for h in range(12):
        q, qs = quant_rows(qkv[:, 32 * h:32 * h + 32], 1.0)
        k, ks = quant_rows(qkv[:, 384 + 32 * h:384 + 32 * h + 32], k_mul)
        v = qkv[:, 768 + 32 * h:768 + 32 * h + 32]
        vm = np.maximum(np.abs(v).max(axis=0), f32(1e-8))
        v_scale = vm * (f32(1.0) / f32(127.0))
        vq = np.clip(np.rint(v * (f32(127.0) / vm)[None, :]), -128, 127).astype(np.int64)
        s = ((q @ k.T).astype(f32) * ks[None, :]) * qs[:, None]
        x = s - s.max(axis=1, keepdims=True)
        xv = np.maximum(x[:, :L8], f32(-16.0))
        n = np.floor(xv).astype(np.int32)
        fr = xv - n.astype(f32)
        p = fma(fr, c[3] * np.ones_like(fr), c[2])
        p = fma(fr, p, c[1])
        p = fma(fr, p, c[0])
        pv = np.rint((p.view(np.int32) + (n << 23)).view(f32)).astype(np.int64)
        e = np.exp2(x[:, L8:]) * f32(16383.0)
        pt = np.clip(np.floor(e.astype(np.float64) + 0.5), 0, 16383).astype(np.int64)
        P = np.concatenate([pv, pt], axis=1)
        p_scale = f32(1.0) / np.maximum(P.sum(axis=1), 1).astype(f32)
        out[:, 32 * h:32 * h + 32] = (P @ vq).astype(f32) * (v_scale[None, :] * p_scale[:, None])
    return out


@pytest.mark.parametrize("L", [1, 4, 16, 33, 128, 512])
def test_int8_attention_restatements_agree(L):
    """The oracle's C++ restatement of the int8 scheme vs an independent NumPy statement, on the
    reference's own benchmark input and on N(0, 1) data."""
    for qkv in (bench_qkv(L), rng(L).normal(0, 1, (L, 1152)).astype(np.float32)):
        got = orc.attention_i8(qkv)
        ref = np_attention_i8(qkv)
        # the only admitted difference: exp2 of the last L % 8 keys (glibc vs NumPy), which can
        # move one 14-bit probability by one step
        assert (got == ref).mean() > 0.99
        np.testing.assert_allclose(got, ref, rtol=0, atol=1e-3 * float(np.abs(ref).max()))
        if L % 8 == 0:
            np.testing.assert_array_equal(got, ref)


def test_int8_attention_mode_forward(pack_path, oracle_model):
    """int8 mode of layers 0-10: sequences under 16 tokens keep the fp32 attention (src/model.rs:245),
    longer ones stay within the reference's own accuracy bar of its int8 path against fp32
    (tests/accuracy_test.rs:109-132: cos > 0.9985 per record); scales are per sequence, so a
    packed batch gives each sequence's single-sequence result."""
    m8 = orc.OracleModel(pack_path).set_attention_mode(orc.ATTENTION_INT8)
    r = rng(77)
    lens = [3, 15, 16, 40, 128, 300]
    seqs = [synth.token_ids(L, r) for L in lens]
    for s in seqs:
        a, b = oracle_model.forward_cls(s), m8.forward_cls(s)
        if len(s) < 16:
            np.testing.assert_array_equal(a, b)
        else:
            assert float(a @ b) > 0.9985 and not np.array_equal(a, b)
    packed = m8.forward_ragged(seqs[:4])
    np.testing.assert_array_equal(packed, np.stack([m8.forward_cls(s) for s in seqs[:4]]))
    with pytest.raises(ValueError):
        m8.set_attention_mode(2)
