"""ae_forward_cls_noalloc: the single-sequence forward for callers that cannot allocate device
memory when they embed (a host that owns every device allocation through its own start-up pool, a
latency path that must not block on cudaMalloc). Its scratch is a static device array inside the
library; this test calls it through the C ABI twice in a row per length and compares each result
with the allocating entry point ae_forward_ragged_device on the same input (identical kernels, so
identical bits). The lengths run short, long, then short again, so a short call also runs on rows
a longer call left behind. The device's free memory must not change across the calls. Named
test_zz_* so that pytest collects it last."""
import ctypes as C

import numpy as np
import pytest
import torch

from arctic_embed_s_int8 import _lib, synth

pytestmark = pytest.mark.gpu


def test_noalloc_matches_allocating_entry_point(engine):
    lib = _lib.lib()
    r = np.random.Generator(np.random.PCG64(77))
    # the first call on a device looks up the static array's address (which may load the library's
    # module and so reserve its memory); free memory is compared from the second call on
    warm = torch.from_numpy(synth.token_ids(8, r).view(np.int16)).cuda()
    sink = torch.zeros(384, dtype=torch.float32, device="cuda")
    _lib.check(engine.handle, lib.ae_forward_cls_noalloc(engine.handle, warm.data_ptr(), 8, sink.data_ptr()))
    engine.sync()
    for L in (33, 512, 17):
        ids = synth.token_ids(L, r)
        d_ids = torch.from_numpy(ids.view(np.int16)).cuda()
        d_cu = torch.tensor([0, L], dtype=torch.int32, device="cuda")
        ref = torch.zeros(1, 384, dtype=torch.float32, device="cuda")
        engine.forward_device(d_ids, d_cu, 1, L, L, ref)
        engine.sync()
        outs = [torch.full((384,), float("nan"), dtype=torch.float32, device="cuda") for _ in range(2)]
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for out in outs:  # two calls in a row on the shared static scratch
            code = lib.ae_forward_cls_noalloc(engine.handle, d_ids.data_ptr(), L, out.data_ptr())
            _lib.check(engine.handle, code)
            engine.sync()
        assert torch.cuda.mem_get_info()[0] == free_before, "the no-alloc entry point changed free device memory"
        for out in outs:
            np.testing.assert_array_equal(out.cpu().numpy(), ref[0].cpu().numpy())


def test_noalloc_rejects_oversize(engine):
    lib = _lib.lib()
    d_ids = torch.zeros(600, dtype=torch.int16, device="cuda")
    out = torch.zeros(384, dtype=torch.float32, device="cuda")
    code = lib.ae_forward_cls_noalloc(engine.handle, d_ids.data_ptr(), 600, out.data_ptr())
    assert code == -7
    assert b"512" in lib.ae_last_error(engine.handle)
    assert lib.ae_forward_cls_noalloc(engine.handle, d_ids.data_ptr(), 0, out.data_ptr()) == -7
