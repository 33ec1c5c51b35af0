"""Row kernels of the forward pass vs the oracle, bit for bit, in the configurations the forward pass
itself runs them in (read back through the ae_trace_forward test hook):

* the embedding rows (dequant_add_embeddings_row, src/simd_math.rs:1827-1881, then
  layernorm_smooth_quantize_row with layers[0].qkv.inv_smooth, src/model.rs:196-219):
  `k_embed_ln_quant`, its LayerNorm output and its int8 rows and scales;
* the quantization of layer 0's attention context for the attention-out GEMM (smooth_quantize_row,
  src/simd_math.rs:584-649): `k_smooth_quant` for packed batches and longer sequences, and the
  quantization inside `k_attention_lat` (12-CTA clusters exchanging row maxima) for single
  sequences of at most 64 tokens. The expected int8 rows are the oracle's quantization of the
  GPU's own context rows; the context rows themselves are checked against the oracle's layer-0
  context at the attention tests' bar.
"""
import numpy as np
import pytest

from arctic_embed_s_int8 import Engine, synth
from conftest import rng
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def _rows(seqs):
    off = 0
    for s in seqs:
        L = min(len(s), 512)
        yield s, slice(off, off + L)
        off += L


@pytest.mark.parametrize("lens", [[1], [8], [32], [129], [512], [700], [2, 7, 128, 33, 512, 1, 64, 300]])
def test_embedding_rows_bit_exact(engine, oracle_model, lens):
    r = rng(400 + sum(lens))
    seqs = [synth.token_ids(L, r) for L in lens]
    hid, q, sc = engine.trace(seqs, Engine.TRACE_EMBED)
    for s, rows in _rows(seqs):
        eh, eq, es = oracle_model.embed_rows(s)
        np.testing.assert_array_equal(hid[rows], eh)
        np.testing.assert_array_equal(q[rows], eq)
        np.testing.assert_array_equal(sc[rows], es)


# single sequences of <= 64 tokens: the attention kernel quantizes the context itself; the others
# (longer single sequences, packed batches) run k_smooth_quant after the attention
@pytest.mark.parametrize("lens", [[1], [8], [32], [33], [64], [65], [128], [512], [3, 64, 17, 128, 40, 250]])
def test_context_quantization_bit_exact(engine, oracle_model, quantized, lens):
    r = rng(500 + sum(lens))
    seqs = [synth.token_ids(L, r) for L in lens]
    ctx, q, sc = engine.trace(seqs, Engine.TRACE_ATTN0)
    eq, es = orc.smooth_quant_rows(ctx, quantized.layers[0].attn_out.inv_smooth)
    np.testing.assert_array_equal(q, eq)
    np.testing.assert_array_equal(sc, es)
    for s, rows in _rows(seqs):
        ref = oracle_model.trace(s)["ctx"][0]
        np.testing.assert_allclose(ctx[rows], ref, rtol=0, atol=2e-6)
        assert (ctx[rows] == ref).mean() > 0.99
