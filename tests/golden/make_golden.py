"""Writes tests/golden/synthetic_seed0.npz: the SHA-256 of the seeded synthetic pack and the CPU
oracle's embeddings of a few token sequences (fp32 attention, and the int8 attention mode). Regenerate only when the synthetic-model recipe or
the oracle changes on purpose:  python tests/golden/make_golden.py"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path[:0] = [ROOT, os.path.join(ROOT, "snowflake-arctic-embed-s-rust_b200")]

from arctic_embed_s_int8 import synth  # noqa: E402
from oracle import oracle as orc  # noqa: E402


def main():
    orc.build()
    path = synth.pack_path(0)
    m = orc.OracleModel(path, orc.BACKEND_AVX2 if orc.lib().or_has_avx2_fma() else orc.BACKEND_SCALAR)
    m8 = orc.OracleModel(path, orc.BACKEND_AVX2 if orc.lib().or_has_avx2_fma() else orc.BACKEND_SCALAR)
    m8.set_attention_mode(orc.ATTENTION_INT8)
    r = np.random.Generator(np.random.PCG64(20251201))
    out = {"pack_sha256": np.array(synth.file_sha256(path))}
    lens = [1, 8, 32, 130]
    for i, L in enumerate(lens):
        ids = synth.token_ids(L, r)
        out[f"ids_{i}"] = ids
        out[f"emb_{i}"] = m.forward_cls(ids)
        out[f"emb_i8_{i}"] = m8.forward_cls(ids)  # the int8 attention mode
    out["n"] = np.array(len(lens))
    np.savez_compressed(os.path.join(os.path.dirname(os.path.abspath(__file__)), "synthetic_seed0.npz"), **out)


if __name__ == "__main__":
    main()
