"""Full forward pass on the B200 vs the CPU oracle on the same seeded synthetic pack and token
ids: cosine >= 0.9999 and max-abs <= 2e-3 on the L2-normalised [CLS] embedding (the north-star
tolerance), for the reference's own length set (tests/parallel_test.rs:21), ragged batches, the
layer-wise int32 accumulators, determinism and the error paths."""
import numpy as np
import pytest
import torch

from conftest import COS_MIN, MAXABS_MAX, REF_LENGTHS, rng
from arctic_embed_s_int8 import AeError, Engine, synth

pytestmark = pytest.mark.gpu


def close(a, b):
    cos = float(np.dot(a, b) / (np.linalg.norm(a) * np.linalg.norm(b)))
    return cos, float(np.abs(a - b).max())


@pytest.mark.parametrize("L", REF_LENGTHS)
def test_forward_cls_matches_oracle(engine, oracle_model, L):
    ids = synth.token_ids(L, rng(1000 + L))
    got = engine.forward_cls(ids)
    ref = oracle_model.forward_cls(ids)
    cos, mx = close(got, ref)
    assert cos >= COS_MIN and mx <= MAXABS_MAX, (L, cos, mx)
    # replayed graph gives the same bits
    np.testing.assert_array_equal(engine.forward_cls(ids), got)


def test_ragged_batch_matches_oracle(engine, oracle_model):
    r = rng(7)
    lens = [1, 2, 3, 8, 12, 16, 31, 64, 100, 128, 200, 333, 512, 5, 1, 77]
    seqs = [synth.token_ids(L, r) for L in lens]
    got = engine.forward_ragged(seqs)
    for s, g in zip(seqs, got):
        cos, mx = close(g, oracle_model.forward_cls(s))
        assert cos >= COS_MIN and mx <= MAXABS_MAX, (len(s), cos, mx)
    # packed == single on the GPU as well
    single = np.stack([engine.forward_cls(s) for s in seqs])
    np.testing.assert_array_equal(got, single)


def test_query_tile_widths_agree(engine, oracle_model):
    """Attention runs in 128-, 64- or 32-query tiles, chosen by how many (sequence, head) pairs a
    launch has. Every width evaluates the same formulas in the same order, so an embedding is the
    same bits whichever width its batch takes: 25 sequences (300 pairs) take 128- / 64-query tiles,
    the same sequences alone (12 pairs) 32-query tiles."""
    r = rng(21)
    for lo, hi in ((97, 128), (33, 64)):
        seqs = [synth.token_ids(int(L), r) for L in r.integers(lo, hi + 1, 25)]
        got = engine.forward_ragged(seqs)
        np.testing.assert_array_equal(engine.forward_ragged(seqs), got)
        for i in (0, 11, 24):
            np.testing.assert_array_equal(engine.forward_cls(seqs[i]), got[i])
        cos, mx = close(got[0], oracle_model.forward_cls(seqs[0]))
        assert cos >= COS_MIN and mx <= MAXABS_MAX, (lo, cos, mx)


def test_fused_and_split_layernorm_paths_agree(engine, oracle_model):
    """A batch of >= 74 row tiles takes the fused LayerNorm GEMM epilogue; a single sequence takes the
    narrow-slice GEMM + LayerNorm row kernel. Both compute the same formulas in the same order, so
    every embedding is bit-identical across the two paths."""
    r = rng(9)
    seqs = [synth.token_ids(512, r) for _ in range(19)] + [synth.token_ids(L, r) for L in (1, 7, 130)]
    assert sum(len(s) for s in seqs) >= 74 * 128
    got = engine.forward_ragged(seqs)
    for i in (0, 7, 18, 19, 20, 21):
        np.testing.assert_array_equal(got[i], engine.forward_cls(seqs[i]))
    cos, mx = close(got[21], oracle_model.forward_cls(seqs[21]))
    assert cos >= COS_MIN and mx <= MAXABS_MAX


def test_reference_ragged_packing(engine, oracle_model):
    """embed_batch packs short sequences (< 16 tokens) into forward_ragged_cls (src/lib.rs:161-238)."""
    r = rng(8)
    seqs = [synth.token_ids(L, r) for L in [5, 9, 3, 12, 7, 2, 15, 4]]
    ref = oracle_model.forward_ragged(seqs[:4])
    got = engine.forward_ragged(seqs[:4])
    for g, o in zip(got, ref):
        cos, mx = close(g, o)
        assert cos >= COS_MIN and mx <= MAXABS_MAX


def test_layerwise_int32_accumulators_bit_exact(engine, oracle_model, quantized):
    """Given the oracle's own int8 activations of every layer, the GPU GEMM reproduces the int32
    accumulators exactly (QKV of layers 0-10, KV-only of layer 11, FFN-down of layers 0-10)."""
    ids = synth.token_ids(48, rng(3))
    tr = oracle_model.trace(ids)
    L = len(ids)
    for l in range(12):
        ly = quantized.layers[l]
        lin = ly.kv_only if l == 11 else ly.qkv
        a = torch.from_numpy(tr["gemm_in_q"][l].copy()).cuda()
        acc = torch.zeros(L, lin.n_out, dtype=torch.int32, device="cuda")
        out = torch.zeros(L, lin.n_out, dtype=torch.float32, device="cuda")
        engine.gemm_i8(0, a, torch.from_numpy(tr["gemm_in_s"][l].copy()).cuda(), torch.from_numpy(lin.w_q).cuda(),
                       torch.from_numpy(lin.w_scale).cuda(), torch.from_numpy(lin.bias).cuda(), out=out, acc=acc)
        engine.sync()
        ref = tr["gemm_in_q"][l].astype(np.int64) @ lin.w_q.astype(np.int64).T
        np.testing.assert_array_equal(acc.cpu().numpy(), ref)
        if l < 11:
            np.testing.assert_array_equal(out.cpu().numpy(), tr["qkv_out"][l])
    for l in range(11):
        lin = quantized.layers[l].ffn_out
        a = torch.from_numpy(tr["down_in_q"][l].copy()).cuda()
        acc = torch.zeros(L, 384, dtype=torch.int32, device="cuda")
        out = torch.zeros(L, 384, dtype=torch.float32, device="cuda")
        engine.gemm_i8(0, a, torch.from_numpy(tr["down_in_s"][l].copy()).cuda(), torch.from_numpy(lin.w_q).cuda(),
                       torch.from_numpy(lin.w_scale).cuda(), torch.from_numpy(lin.bias).cuda(), out=out, acc=acc)
        engine.sync()
        np.testing.assert_array_equal(acc.cpu().numpy(), tr["down_in_q"][l].astype(np.int64) @ lin.w_q.astype(np.int64).T)


def test_fresh_engines_deterministic(pack_path):
    """Regression idea of tests/parallel_test.rs:54-64: the first call on a fresh context completes
    and is bit-identical to another fresh context's."""
    ids = synth.token_ids(33, rng(5))
    e1 = Engine(0).load_file(pack_path)
    e2 = Engine(0).load_file(pack_path)
    a, b = e1.forward_cls(ids), e2.forward_cls(ids)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(e1.forward_ragged([ids])[0], a)
    e1.close()
    e2.close()


def test_model_reload(pack_path):
    """QuantizedModelRaw::load_ae8 + PackedModel::from_raw (src/quantize.rs:76-137, src/model.rs:49-84)
    run again on a live context: a reload of the same model shape reuses the device arena, and the
    single-sequence graphs captured before it then compute with the new weights; the host-array
    descriptor path (ae_model_load) gives the same bits as the file path."""
    from arctic_embed_s_int8 import ae8

    other = synth.pack_path(1)
    ids = synth.token_ids(40, rng(13))
    e = Engine(0).load_file(pack_path)
    a0 = e.forward_cls(ids)
    e.load_file(other)
    b = e.forward_cls(ids)
    fresh = Engine(0).load_file(other)
    np.testing.assert_array_equal(b, fresh.forward_cls(ids))
    assert not np.array_equal(a0, b)
    e.load(ae8.read_ae8(pack_path))
    np.testing.assert_array_equal(e.forward_cls(ids), a0)
    np.testing.assert_array_equal(e.forward_ragged([ids, ids[:7]])[0], a0)
    e.load_file(pack_path)
    np.testing.assert_array_equal(e.forward_cls(ids), a0)
    # a short sequence (the single-kernel cluster forward) across a reload of other weights
    short = synth.token_ids(20, rng(14))
    s0 = e.forward_cls(short)
    e.load_file(other)
    np.testing.assert_array_equal(e.forward_cls(short), fresh.forward_cls(short))
    e.load_file(pack_path)
    np.testing.assert_array_equal(e.forward_cls(short), s0)
    fresh.close()
    e.close()


def test_cluster_forward_matches_multi_kernel_path(pack_path, oracle_model, monkeypatch):
    """Single sequences of at most 32 tokens run as one 12-CTA cluster kernel (latency.cu); it
    computes every value with the multi-kernel path's arithmetic in the same order, so every
    embedding is the same bits (ARCTIC_LAT_CLUSTER=0 selects the multi-kernel path), one launch per
    forward instead of about 90, and within the tolerance of the oracle."""
    monkeypatch.setenv("ARCTIC_LAT_CLUSTER", "0")
    multi = Engine(0).load_file(pack_path)
    monkeypatch.delenv("ARCTIC_LAT_CLUSTER")
    one = Engine(0).load_file(pack_path)
    r = rng(77)
    for L in range(1, 33):
        for _ in range(2 if L in (1, 8, 16, 17, 31, 32) else 1):
            ids = synth.token_ids(L, r)
            n0 = one.kernel_launches()
            got = one.forward_cls(ids)
            assert one.kernel_launches() - n0 == 1, L
            np.testing.assert_array_equal(got, multi.forward_cls(ids), err_msg=f"L={L}")
    for L in (3, 32):  # against the oracle as well
        ids = synth.token_ids(L, r)
        cos, mx = close(one.forward_cls(ids), oracle_model.forward_cls(ids))
        assert cos >= COS_MIN and mx <= MAXABS_MAX, (L, cos, mx)
    # longer sequences keep the multi-kernel path
    ids = synth.token_ids(33, r)
    n0 = one.kernel_launches()
    np.testing.assert_array_equal(one.forward_cls(ids), multi.forward_cls(ids))
    assert one.kernel_launches() - n0 > 1
    multi.close()
    one.close()


def test_truncation_to_512(engine):
    ids = synth.token_ids(700, rng(6))
    np.testing.assert_array_equal(engine.forward_cls(ids), engine.forward_cls(ids[:512]))
    got = engine.forward_ragged([ids, ids[:10]])
    np.testing.assert_array_equal(got[0], engine.forward_cls(ids[:512]))


def test_error_paths(engine, pack_path):
    with pytest.raises(AeError, match="TOKEN_RANGE"):
        engine.forward_cls(np.array([101, 30522, 102], np.uint16))
    with pytest.raises(AeError, match="INVALID_ARG"):
        engine.forward_cls(np.zeros(0, np.uint16))
    with pytest.raises(AeError, match="INVALID_ARG"):
        engine.forward_ragged([np.array([101, 102], np.uint16), np.zeros(0, np.uint16)])
    e = Engine(0)
    with pytest.raises(AeError, match="NO_MODEL"):
        e.forward_cls(np.array([101, 102], np.uint16))
    with pytest.raises(AeError, match="BAD_PACK"):
        e.load_file(pack_path + ".missing")
    e.close()
    # the engine still works after the errors
    assert np.isfinite(engine.forward_cls(np.array([101, 2000, 102], np.uint16))).all()


def test_device_resident_forward(engine):
    r = rng(11)
    seqs = [synth.token_ids(L, r) for L in [128] * 8 + [3, 500]]
    from arctic_embed_s_int8 import pack_sequences

    ids, cu = pack_sequences(seqs)
    d_ids = torch.from_numpy(ids.view(np.int16)).cuda()
    d_cu = torch.from_numpy(cu.view(np.int32)).cuda()
    out = torch.zeros(len(seqs), 384, dtype=torch.float32, device="cuda")
    engine.forward_device(d_ids, d_cu, len(seqs), int(cu[-1]), 512, out)
    engine.sync()
    np.testing.assert_array_equal(out.cpu().numpy(), engine.forward_ragged(seqs))


def test_text_to_embedding(engine, oracle_model):
    """embed_query / embed_document / embed_batch (src/lib.rs:96-260): the C++ WordPiece tokenizer
    feeding the GPU forward; ids identical to the reference's known answers, embeddings within the
    tolerance of the oracle on the same ids, batch == one at a time."""
    from conftest import golden_vocab_text
    from arctic_embed_s_int8 import ArcticEmbedS
    from arctic_embed_s_int8.tokenizer import BertTokenizer

    vocab, records = golden_vocab_text()
    model = ArcticEmbedS(engine, tokenizer=BertTokenizer.from_vocab_str(vocab))
    picked = [r for r in records if r["kind"] == "query"][:3] + [r for r in records if r["kind"] == "document"][-2:]
    for r in picked:
        got = model.embed_query(r["text"]) if r["kind"] == "query" else model.embed_document(r["text"])
        cos, mx = close(got, oracle_model.forward_cls(np.array(r["ids"], np.uint16)))
        assert cos >= COS_MIN and mx <= MAXABS_MAX, (r["text"][:40], cos, mx)
    docs = [r["text"] for r in records if r["kind"] == "document"]
    batch = model.embed_batch(docs)
    for t, b in zip(docs, batch):
        np.testing.assert_array_equal(b, model.embed_document(t))


def test_bounded_wait_reports_error(engine):
    """Failure detection without a GPU fault: a device wait that can never complete gives up after
    its limit, the host gets AE_ERR_DEVICE with the reason, and the context keeps working."""
    with pytest.raises(AeError, match="DEVICE.*timed out"):
        engine.selftest_wait_timeout(2000)
    ids = synth.token_ids(20, rng(12))
    np.testing.assert_array_equal(engine.forward_cls(ids), engine.forward_cls(ids))
    engine.sync()


def test_fused_qkv_attention_matches_split(pack_path, oracle_model, monkeypatch):
    """The QKV projection fused into the attention kernel (sequences of at most 128 keys) computes the
    QKV GEMM's dequantization and the attention in the same order as the split path (GEMM to global
    memory, then the attention kernels), so every embedding is the same bits. ARCTIC_FUSED_QKV forces
    either path at context creation; sequences start at unaligned rows and run past tile ends."""
    r = rng(31)
    batches = [[synth.token_ids(128, r) for _ in range(30)],
               [synth.token_ids(int(L), r) for L in r.integers(1, 129, 40)],
               [synth.token_ids(L, r) for L in (1, 2, 3, 4, 5, 31, 32, 33, 63, 64, 65, 127, 128)]]
    engines = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("ARCTIC_FUSED_QKV", mode)
        engines[mode] = Engine(0).load_file(pack_path)
    monkeypatch.delenv("ARCTIC_FUSED_QKV")
    for seqs in batches:
        split = engines["0"].forward_ragged(seqs)
        fused = engines["1"].forward_ragged(seqs)
        np.testing.assert_array_equal(fused, split)
    for L in (1, 17, 64, 100, 128):
        ids = synth.token_ids(L, rng(300 + L))
        got = engines["1"].forward_cls(ids)
        np.testing.assert_array_equal(got, engines["0"].forward_cls(ids))
        cos, mx = close(got, oracle_model.forward_cls(ids))
        assert cos >= COS_MIN and mx <= MAXABS_MAX, (L, cos, mx)
    for e in engines.values():
        e.close()


def test_few_long_sequence_attention_matches_tmem_kernels(pack_path, oracle_model, monkeypatch):
    """Few (sequence, head) pairs of more than 64 keys (single sequences of 65-512 tokens, small
    batches) run the attention either on 32-query tiles with the scores in shared memory or with
    eight lanes per query, whichever fills the SMs in one wave. Both keep every chain of the
    reference's order in one thread, so every embedding is the same bits as with the TMEM kernels
    (ARCTIC_ATTN_FEW=tmem; =narrow, =lanes8 and =dm force the others at every length; dm is the
    32-query-tile kernel with K / V staged dim-major, by bulk copies when the sequence starts a
    128-row tile, the single-sequence default), and within the tolerance of the oracle."""
    engines = {}
    for mode in ("tmem", "narrow", "lanes8", "dm", None):
        if mode:
            monkeypatch.setenv("ARCTIC_ATTN_FEW", mode)
        else:
            monkeypatch.delenv("ARCTIC_ATTN_FEW")
        engines[mode] = Engine(0).load_file(pack_path)
    tmem = engines.pop("tmem")
    r = rng(88)
    for L in (65, 66, 97, 100, 127, 128, 129, 130, 200, 255, 256, 257, 300, 383, 384, 385, 500, 511, 512):
        ids = synth.token_ids(L, r)
        ref = tmem.forward_cls(ids)
        for mode, e in engines.items():
            np.testing.assert_array_equal(e.forward_cls(ids), ref, err_msg=f"{mode} L={L}")
    for lens in ([70, 128], [512, 129, 300], [100] * 12, [90, 3, 65, 128, 77]):
        seqs = [synth.token_ids(L, r) for L in lens]
        ref = tmem.forward_ragged(seqs)
        for mode, e in engines.items():
            np.testing.assert_array_equal(e.forward_ragged(seqs), ref, err_msg=f"{mode} {lens}")
    for L in (65, 512):
        ids = synth.token_ids(L, r)
        cos, mx = close(engines[None].forward_cls(ids), oracle_model.forward_cls(ids))
        assert cos >= COS_MIN and mx <= MAXABS_MAX, (L, cos, mx)
    tmem.close()
    for e in engines.values():
        e.close()
