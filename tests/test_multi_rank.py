"""Multi-rank host logic on CPU (gloo, world_size 2): row sharding of a global
batch, each rank's slice of the reference uniform stream, and the
max-over-ranks timing that bench.py uses under torchrun.

Rows are independent (src/model.c:1268-1307 samples one logits row at a
time), so a sharded batch must give exactly the ids of the unsharded one; the
oracle stands in for the per-rank sampler here.
"""
import os
import socket
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")]

import bench  # noqa: E402

TOTAL = 18  # not a multiple of the world size: ragged shards


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch():
    import synth
    return synth.make_c4(77, TOTAL, V=3001, Hmax=200)


def _rank_main(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist

    import oracle
    import synth
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        b = _batch()
        start, count = bench.shard_rows(TOTAL, world, rank)
        u = bench.ref_uniforms(TOTAL)[start:start + count]
        sl = slice(start, start + count)
        off = b.hist_off[start:start + count + 1] - b.hist_off[start]
        mine = synth.Batch(b.logits[sl], b.hist[b.hist_off[start]:b.hist_off[start + count]],
                           off, b.temp[sl], b.penalty[sl], b.min_p[sl], b.top_p[sl],
                           b.top_k[sl])
        ids, _, _ = oracle.sample_batch(mine, u)
        m = bench.max_over_ranks(dist, 1.5 + rank)
        np.save(os.path.join(out_dir, f"r{rank}.npy"),
                np.concatenate([[start, count], ids.astype(np.int64), [int(m * 10)]]))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_shard_rows_tile_the_batch():
    for total in (0, 1, 7, 4096 * 8, 4097):
        for world in (1, 2, 3, 8):
            spans = [bench.shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0
            for (s0, c0), (s1, _) in zip(spans, spans[1:]):
                assert s0 + c0 == s1
            assert sum(c for _, c in spans) == total
            assert max(c for _, c in spans) - min(c for _, c in spans) <= 1


def test_max_over_ranks_single_process():
    assert bench.max_over_ranks(None, 3.25) == 3.25


def test_two_rank_gloo_shards_match_unsharded(tmp_path):
    import torch.multiprocessing as mp

    import oracle
    oracle.lib()  # build/load before the ranks start
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    got = {}
    for r in range(world):
        a = np.load(tmp_path / f"r{r}.npy")
        start, count = int(a[0]), int(a[1])
        got[start] = a[2:2 + count]
        assert a[-1] == 25  # max over ranks of 1.5 + rank, x10
    sharded = np.concatenate([got[k] for k in sorted(got)])
    b = _batch()
    whole, _, _ = oracle.sample_batch(b, bench.ref_uniforms(TOTAL))
    assert np.array_equal(sharded, whole)


if __name__ == "__main__":
    sys.exit(pytest.main([__file__, "-q"]))
