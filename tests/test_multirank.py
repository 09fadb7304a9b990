"""The N-rank layout of bench.py on CPU ranks (gloo, world size 2): the batched job's
sequence partition (i mod world == rank) serves each of the 512 sequences exactly once,
the per-rank results gathered over the host group add up to the one-rank job's totals,
and the reported time is the maximum over the ranks.  The data path has no collective;
the group only carries the barrier and the gather of the results."""
import json
import multiprocessing as mp
import os
import socket
import sys
import types

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
JOB = 512


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_path):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, ROOT)
    import bench

    group = bench.Group()
    mine = bench.partition(JOB, group.world, group.rank)
    group.barrier()
    # stand-in results of this rank's share: one first token per sequence plus 3 more,
    # and a rank-dependent decode time
    res = {"nseq": len(mine), "generated": 4 * len(mine), "decode_s": 1.0 + rank, "wall": 2.0 + rank,
           "launches": 196, "seqs": mine}
    gathered = group.gather(res)
    if group.rank == 0:
        with open(out_path, "w") as f:
            json.dump(gathered, f)
    group.close()


def _run(world, tmp_path):
    port = _free_port()
    out = str(tmp_path / f"gathered{world}.json")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    with open(out) as f:
        return json.load(f)


def test_partition_covers_each_sequence_once():
    sys.path.insert(0, ROOT)
    import bench
    for world in (1, 2, 4, 8):
        shares = [bench.partition(JOB, world, r) for r in range(world)]
        served = sorted(i for s in shares for i in s)
        assert served == list(range(JOB))
        assert max(map(len, shares)) - min(map(len, shares)) <= 1


def test_two_gloo_ranks_gather_the_one_rank_totals(tmp_path):
    sys.path.insert(0, ROOT)
    import bench

    two = _run(2, tmp_path)
    one = _run(1, tmp_path)
    assert sorted(i for g in two for i in g["seqs"]) == list(range(JOB))
    assert sum(g["generated"] for g in two) == sum(g["generated"] for g in one)
    assert sum(g["nseq"] for g in two) == sum(g["nseq"] for g in one) == JOB
    args = types.SimpleNamespace(serve_new=4, serve_seqs=JOB)
    obj2 = bench.batched_object(two, args, 2)
    obj1 = bench.batched_object(one, args, 1)
    assert obj2["decode_s"] == 2.0          # the slower rank's time
    assert obj2["value"] == (4 * JOB - JOB) / 2.0
    assert obj1["value"] == (4 * JOB - JOB) / 1.0
