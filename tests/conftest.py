"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on the CPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "snowflake-arctic-embed-s-rust_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

# sequence lengths of the reference's parallel test (tests/parallel_test.rs:21), plus 32: the parity
# configuration (one 32-token sequence)
REF_LENGTHS = [1, 2, 5, 8, 15, 16, 17, 31, 32, 33, 64, 100, 128, 257, 512]
COS_MIN = 0.9999     # north-star tolerance on the final embeddings
MAXABS_MAX = 2e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA library)")


@pytest.fixture(scope="session")
def pack_path():
    from arctic_embed_s_int8 import synth

    return synth.pack_path(0)


@pytest.fixture(scope="session")
def oracle_model(pack_path):
    from oracle import oracle as orc

    orc.build()
    return orc.OracleModel(pack_path)


@pytest.fixture(scope="session")
def quantized(pack_path):
    from arctic_embed_s_int8 import ae8

    return ae8.read_ae8(pack_path)


@pytest.fixture(scope="session")
def engine(pack_path):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a GPU")
    from arctic_embed_s_int8 import Engine

    eng = Engine(0).load_file(pack_path)
    yield eng
    eng.close()


def rng(seed=0):
    return np.random.Generator(np.random.PCG64(seed))


def golden_vocab_text() -> tuple:
    """(vocabulary text, records) of the tokenizer fixture: the full id space with the golden subset at its ids and a
    control character (removed by the normalizer, so never matched) on every other line."""
    import json

    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tokenizer_vectors.json"),
              encoding="utf-8") as f:
        g = json.load(f)
    sub = g["vocab_subset"]
    return "\n".join(sub.get(str(i), f"\x01{i}") for i in range(g["vocab_size"])) + "\n", g["records"]
