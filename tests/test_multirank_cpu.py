"""The N>1 path on the CPU: two gloo ranks each embed the shard the planner gives them (with the
oracle standing in for the GPU engine), then gather; the result equals the single-process result.
This is the plumbing bench.py and ae_embed_batch_multi use: shards with no data-path collective,
outputs gathered by index."""
import os
import socket

import numpy as np
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, pack, ids, cu, out_path):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "snowflake-arctic-embed-s-rust_b200")]
    import torch
    import torch.distributed as dist

    from arctic_embed_s_int8 import plan_shards
    from oracle import oracle as orc

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shard = plan_shards(cu, world)
    mine = np.nonzero(shard == rank)[0]
    m = orc.OracleModel(pack)
    out = np.zeros((len(cu) - 1, 384), np.float32)
    for i in mine:
        out[i] = m.forward_cls(ids[cu[i]:cu[i + 1]])
    t = torch.from_numpy(out)
    dist.all_reduce(t)  # disjoint rows: the sum is the gather
    if rank == 0:
        np.save(out_path, t.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_gloo_sharding(pack_path, oracle_model, tmp_path):
    from arctic_embed_s_int8 import pack_sequences, synth

    r = np.random.Generator(np.random.PCG64(2))
    seqs = [synth.token_ids(int(L), r) for L in r.integers(2, 60, 10)]
    ids, cu = pack_sequences(seqs)
    out_path = str(tmp_path / "out.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(k, 2, port, pack_path, ids, cu, out_path)) for k in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = np.load(out_path)
    ref = oracle_model.embed_batch(seqs, 2)
    np.testing.assert_array_equal(got, ref)
