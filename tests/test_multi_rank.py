"""Host logic of the multi-device paths on CPU (gloo, ranks as separate processes): both merges of the sharded stage
(by collectives: maxima all-reduced, states scaled to them and summed, each rank keeping its equal slice of the
padded rows; by peer stores: every rank's states of a row sent to the rank owning it and merged there in rank order)
give the attention over the whole cache; the shards cover every training row once. The same protocols run on GPUs
in tests/test_gpu_multi.py."""
import json
import os
import socket
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(mode, world, timeout, env=None):
    port = free_port()
    procs = [subprocess.Popen([sys.executable, os.path.join(HERE, "multi_rank.py"), mode, str(r), str(world), str(port)],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True, env=env)
             for r in range(world)]
    outs = []
    try:
        for p in procs:
            o, e = p.communicate(timeout=timeout)
            assert p.returncode == 0, e[-3000:]
            outs.append(json.loads(o.strip().splitlines()[-1]))
    finally:
        for p in procs:
            if p.poll() is None:
                p.kill()
    return outs


@pytest.mark.parametrize("world", [2, 3])
def test_merge_over_ranks_equals_whole_cache(world):
    outs = run_ranks("merge-cpu", world, timeout=120)
    for o in outs:
        assert o["err"] < 1e-12, o
        assert o["rows_total"] == 333 and o["test_rows_total"] == 7
    assert sum(o["rows"] for o in outs) == 333


@pytest.mark.parametrize("world", [2, 3])
def test_merge_by_peer_stores_equals_whole_cache(world):
    outs = run_ranks("push-cpu", world, timeout=120)
    for o in outs:
        assert o["err"] < 1e-12, o


@pytest.mark.parametrize("n,world", [(1, 1), (7, 2), (40, 3), (39, 8), (3, 8)])
def test_shard_chunks_cover_each_chunk_once(n, world):
    sys.path.insert(0, HERE)
    from conftest import load_package
    tcu = load_package()
    seen = []
    for r in range(world):
        first, count = tcu.shard_chunks(n, world, r)
        seen.extend(range(first, first + count))
    assert seen == list(range(n))
