"""The C-ABI library: loads without a GPU, exports every function include/arctic_cuda.h declares,
and reports errors through return codes instead of crashing. No compute calls (no GPU here)."""
import os
import re
import subprocess

import numpy as np
import pytest

from arctic_embed_s_int8 import _lib, plan_shards, pack_sequences

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "arctic_cuda.h")


def declared():
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(ae_[a-z_0-9]+)\s*\(", txt)))


def test_header_and_binding_agree():
    assert declared() == sorted(_lib.SYMBOLS)


def test_library_exports_every_symbol():
    lib = _lib.lib()
    for name in declared():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (ae_\w+)", out))
    assert set(declared()) <= exported


def test_errors_are_codes_not_crashes():
    import ctypes as C

    lib = _lib.lib()
    h = C.c_void_p()
    code = lib.ae_ctx_create(0, C.byref(h))
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if not has_gpu:
        assert code == -2 and not h.value
        assert lib.ae_last_error(None)
    else:
        assert code == 0
        lib.ae_ctx_destroy(h)
    assert lib.ae_ctx_create(0, None) == -1
    assert lib.ae_sync(None) == -1
    assert lib.ae_forward_cls(None, None, 0, None) == -1
    assert lib.ae_set_attention_mode(None, 1) == -1
    assert lib.ae_get_attention_mode(None) == -1
    assert lib.ae_attention_i8(None, None, None, 1, 16, None) == -1


def test_plan_shards_balances_cost():
    r = np.random.Generator(np.random.PCG64(0))
    lens = np.exp(r.uniform(np.log(8), np.log(512), 5000)).astype(int)
    _, cu = pack_sequences([np.full(L, 101, np.uint16) for L in lens])
    for k in (1, 2, 4, 8):
        shard = plan_shards(cu, k)
        assert shard.min() == 0 and shard.max() == k - 1
        L = np.minimum(lens, 512).astype(np.float64)
        cost = 19759104.0 * L + 8448.0 * L * L
        loads = np.array([cost[shard == d].sum() for d in range(k)])
        assert loads.max() / loads.mean() < 1.01
    with pytest.raises(_lib.AeError):
        plan_shards(np.array([0, 5, 3], np.uint32), 2)
