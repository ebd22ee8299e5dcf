"""The N>1 host logic of bench.py on CPU ranks (gloo, world size 2): expert-parallel placement (every
expert id of a layer lands on exactly one rank, id mod world size), the max-over-ranks timing, the sum of
per-rank counters and the all-gather of the per-record outcome table."""
import multiprocessing as mp
import os
import socket
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        sys.path.insert(0, ROOT)
        import datetime

        import torch.distributed as dist
        import bench
        dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
        cfg = dict(bench.CONFIGS['mid'], layers=4)
        trace = bench.routing_trace(cfg, 3, rank, world, cfg['layers'])
        ids = [int(e) for step in trace for layer in step for e in layer]
        rows = [(rank, l, int(e), 0, '') for s, step in enumerate(trace) for l, layer in enumerate(step) for e in layer]
        table = bench.gather_outcomes(rows, world)
        out = {
            'own_shard': all(i % world == rank for i in ids),
            'distinct_per_layer': all(len(set(map(int, layer))) == len(layer) for step in trace for layer in step),
            'max': bench.max_over_ranks(10.0 + rank, world),
            'sum': bench.sum_over_ranks([1.0, float(len(ids))], world),
            'table': table,
        }
        bench.barrier(world)
        dist.destroy_process_group()
        q.put((rank, out))
    except Exception as e:   # reported to the parent, which fails the test
        q.put((rank, repr(e)))


def test_two_cpu_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context('spawn')
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert isinstance(results[r], dict), results[r]
        assert results[r]['own_shard'] and results[r]['distinct_per_layer']
        assert results[r]['max'] == 11.0
    n0 = results[0]['sum'][1]
    assert results[0]['sum'] == results[1]['sum'] and results[0]['sum'][0] == 2.0
    table = results[0]['table']
    assert table == results[1]['table'] and len(table) == n0
    # every rank decodes only its shard: no (layer, expert) pair appears on two ranks
    owner = {}
    for rank, layer, expert, _, _ in table:
        assert owner.setdefault((layer, expert), rank) == rank
    assert {r for r, *_ in table} == {0, 1}


def test_streaming_trace_covers_every_expert_once_per_step():
    """The whole-box config: each rank decodes all of its shard every step, and the shards of all ranks
    partition the experts of every layer."""
    sys.path.insert(0, ROOT)
    import bench
    cfg = bench.CONFIGS['box']
    for world in (1, 2, 8):
        seen = {}
        for rank in range(world):
            trace = bench.routing_trace(cfg, 2, rank, world, cfg['layers'])
            assert trace[0] == trace[1]
            for l, layer in enumerate(trace[0]):
                assert all(e % world == rank for e in layer)
                for e in layer:
                    assert seen.setdefault((l, e), rank) == rank
        assert len(seen) == cfg['layers'] * cfg['experts']
