"""ae_embed_batch_multi: sequences sharded over every visible GPU (and over two contexts on one GPU)
give, in input order, the same bits as one context running them all (rows are independent)."""
import numpy as np
import pytest
import torch

from conftest import rng
from arctic_embed_s_int8 import Engine, embed_batch_multi, synth

pytestmark = pytest.mark.gpu


def test_sharded_equals_single(engine, pack_path):
    r = rng(21)
    lens = np.exp(r.uniform(np.log(2), np.log(600), 300)).astype(int)
    seqs = [synth.token_ids(int(L), r) for L in lens]
    ref = engine.forward_ragged(seqs)
    n_dev = torch.cuda.device_count()
    engines = [Engine(d).load_file(pack_path) for d in range(n_dev)]
    if n_dev == 1:
        engines.append(Engine(0).load_file(pack_path))  # two contexts sharing one GPU
    got = embed_batch_multi(engines, seqs=seqs, max_batch_tokens=8192)
    np.testing.assert_array_equal(got, ref)
    for e in engines:
        e.close()
