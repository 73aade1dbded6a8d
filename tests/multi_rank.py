"""One rank of a multi-process test (run by tests/test_multi_rank.py and tests/test_gpu_multi.py as subprocesses).

    python tests/multi_rank.py MODE RANK WORLD PORT

MODE
  merge-cpu  gloo on CPU: the cross-device merge of the sharded stage (maxima all-reduced, states scaled to them,
             summed with each rank keeping its slice of rows, divided) on shards of a random cache, in numpy,
             against attention over the whole cache (src/nn.rs:187-286).
  push-cpu   gloo on CPU: the same merge by peer stores (every rank's states of a row to the rank owning the row,
             merged there in rank order).
  stage-gpu  one GPU per rank: the sharded stage through the C ABI against the oracle's stage over the whole
             cache, and the f64 all-reduce of ensemble members' class-logit sums.
Prints one JSON line with the rank's result.
"""
import json
import os
import sys
from datetime import timedelta

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def init(rank, world, port):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60))
    return dist


def shard_chunks(nchunks, world, rank):
    base, extra = divmod(nchunks, world)
    return rank * base + min(rank, extra), base + (1 if rank < extra else 0)


def merge_cpu(rank, world, port):
    """The merge of the sharded stage: each rank's unnormalised state per (row, head) over its chunks; the maxima
    all-reduced (max); each rank's states scaled to them; summed over ranks and each rank keeping its slice of rows
    (a reduce-scatter: here an all-reduce of the sum, then the slice); divided (nn.rs:261-286). The rows are padded to
    equal slices."""
    import torch
    dist = init(rank, world, port)
    rng = np.random.default_rng(7)
    R, H, hd, n, chunk = 7, 4, 16, 333, 40
    d = H * hd
    Rs = -(-R // world)
    q = np.zeros((Rs * world, d))
    q[:R] = rng.normal(0, 1, (R, d))
    k = rng.normal(0, 1, (n, d))
    v = rng.normal(0, 1, (n, d))
    nchunks = (n + chunk - 1) // chunk
    c0, nc = shard_chunks(nchunks, world, rank)
    lo, hi = c0 * chunk, min(n, (c0 + nc) * chunk)
    m_loc = np.zeros((len(q), H))
    packed = np.zeros((len(q), d + H))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        sc = q[:, sl] @ k[lo:hi, sl].T
        m = sc.max(1)
        p = np.exp(sc - m[:, None])
        m_loc[:, h] = m
        packed[:, sl] = p @ v[lo:hi, sl]
        packed[:, d + h] = p.sum(1)
    mt = torch.from_numpy(m_loc.copy())
    dist.all_reduce(mt, op=dist.ReduceOp.MAX)
    w = np.exp(m_loc - mt.numpy())
    for h in range(H):
        packed[:, h * hd:(h + 1) * hd] *= w[:, h:h + 1]
        packed[:, d + h] *= w[:, h]
    pt = torch.from_numpy(packed)
    dist.all_reduce(pt, op=dist.ReduceOp.SUM)
    mine = pt.numpy()[rank * Rs:(rank + 1) * Rs]
    att = np.concatenate([mine[:, h * hd:(h + 1) * hd] / mine[:, d + h:d + h + 1] for h in range(H)], 1)
    want = np.zeros((len(q), d))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        sc = q[:, sl] @ k[:, sl].T
        p = np.exp(sc - sc.max(1, keepdims=True))
        want[:, sl] = (p / p.sum(1, keepdims=True)) @ v[:, sl]
    real = max(0, min(Rs, R - rank * Rs))
    counts = torch.tensor([hi - lo, real])
    dist.all_reduce(counts)
    dist.destroy_process_group()
    return {"rank": rank, "err": float(np.abs(att - want[rank * Rs:(rank + 1) * Rs]).max()), "rows_total": int(counts[0]),
            "rows": hi - lo, "test_rows_total": int(counts[1])}


def push_cpu(rank, world, port):
    """The merge of the sharded stage by peer stores: each rank's unnormalised state per (row, head) over its chunks,
    for the rows of rank j's slice, goes to rank j (here by send/receive), which merges every rank's states in rank
    order (nn.rs:261-286: the largest maximum, each state scaled to it, the sums, the division). Rows padded to equal
    slices."""
    import torch
    dist = init(rank, world, port)
    rng = np.random.default_rng(9)
    R, H, hd, n, chunk = 7, 2, 8, 200, 24
    d = H * hd
    Rs = -(-R // world)
    q = np.zeros((Rs * world, d))
    q[:R] = rng.normal(0, 1, (R, d))
    k = rng.normal(0, 1, (n, d))
    v = rng.normal(0, 1, (n, d))
    c0, nc = shard_chunks((n + chunk - 1) // chunk, world, rank)
    lo, hi = c0 * chunk, min(n, (c0 + nc) * chunk)
    ms = np.zeros((len(q), H, 2))
    acc = np.zeros((len(q), d))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        sc = q[:, sl] @ k[lo:hi, sl].T
        m = sc.max(1)
        p = np.exp(sc - m[:, None])
        ms[:, h, 0], ms[:, h, 1] = m, p.sum(1)
        acc[:, sl] = p @ v[lo:hi, sl]
    got_ms = np.zeros((world, Rs, H, 2))
    got_acc = np.zeros((world, Rs, d))
    reqs, bufs = [], []
    for j in range(world):
        part = slice(j * Rs, (j + 1) * Rs)
        if j == rank:
            got_ms[j], got_acc[j] = ms[part], acc[part]
            continue
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(ms[part])), j, tag=0))
        reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(acc[part])), j, tag=1))
        bm, ba = torch.zeros((Rs, H, 2), dtype=torch.float64), torch.zeros((Rs, d), dtype=torch.float64)
        reqs.append(dist.irecv(bm, j, tag=0))
        reqs.append(dist.irecv(ba, j, tag=1))
        bufs.append((j, bm, ba))
    for r in reqs:
        r.wait()
    for j, bm, ba in bufs:
        got_ms[j], got_acc[j] = bm.numpy(), ba.numpy()
    att = np.zeros((Rs, d))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        M = got_ms[:, :, h, 0].max(0)
        w = np.where(got_ms[:, :, h, 1] > 0, np.exp(got_ms[:, :, h, 0] - M), 0.0)
        S = (got_ms[:, :, h, 1] * w).sum(0)
        att[:, sl] = (got_acc[:, :, sl] * w[:, :, None]).sum(0) / S[:, None]
    want = np.zeros((len(q), d))
    for h in range(H):
        sl = slice(h * hd, (h + 1) * hd)
        sc = q[:, sl] @ k[:, sl].T
        p = np.exp(sc - sc.max(1, keepdims=True))
        want[:, sl] = (p / p.sum(1, keepdims=True)) @ v[:, sl]
    dist.destroy_process_group()
    return {"rank": rank, "err": float(np.abs(att - want[rank * Rs:(rank + 1) * Rs]).max())}


def stage_gpu(rank, world, port):
    import torch
    sys.path.insert(0, HERE)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from conftest import load_package
    tcu = load_package()
    from tabicl_anywhere_b200 import synth
    import oracle
    dist = init(rank, world, port)
    torch.cuda.set_device(rank)
    gpu = tcu.Gpu(rank)
    uid = torch.zeros(tcu.COMM_ID_BYTES, dtype=torch.uint8)
    if rank == 0:
        uid = torch.frombuffer(bytearray(tcu.comm_unique_id()), dtype=torch.uint8)
    dist.broadcast(uid, 0)
    comm = tcu.Comm(gpu, bytes(uid.numpy().tobytes()), world, rank)
    out = {"rank": rank, "stage": {}}
    for kv in (1, 2):
        cfg = synth.config("full", icl_num_blocks=2)
        wt = synth.weights(cfg, seed=30 + kv, std=0.08)
        m = oracle.Model({k: v for k, v in wt.items() if k.startswith("icl_predictor.")}, cfg["icl_nhead"], 2,
                         cfg["max_classes"])
        n, chunk = 1500, 256
        caches, scales = oracle.icl_fit(m, synth.row_reps(n, m.d, 31), synth.labels(n, 10, 32), chunk, kv)
        w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")})
        full = tcu.VramModel.from_parts(w, [n, 7, 10, chunk, kv, 1, 1], n, 10, scales, caches)
        c0, nc = tcu.shard_chunks((n + chunk - 1) // chunk, world, rank)
        shard = full.slice(c0, nc)
        for rows in (1, 5, 70, 301, 8200):
            h = synth.row_reps(rows, m.d, 40 + rows)
            hd_ = torch.from_numpy(h).cuda()
            o = torch.empty((rows, 10), device="cuda")
            shard.stage_sharded_device(comm, hd_.data_ptr(), rows, 10, o.data_ptr(), torch.cuda.current_stream().cuda_stream)
            comm.wait(30000, torch.cuda.current_stream().cuda_stream)
            got = o.cpu().numpy()
            want = oracle.in_context(m, kv, caches, scales, n, chunk, h, 10)
            out["stage"][f"kv{kv}_r{rows}"] = float(np.abs(got - want).max())
        shard.free(), full.free(), w.free()
    # ensemble members one per device: each rank's member logit sums, summed over ranks in f64
    sums = torch.full((6, 3), float(rank + 1), dtype=torch.float64, device="cuda")
    comm.allreduce_f64(sums.data_ptr(), sums.numel(), torch.cuda.current_stream().cuda_stream)
    comm.wait(30000, torch.cuda.current_stream().cuda_stream)
    out["allreduce_f64"] = float(sums[0, 0].item())
    torch.cuda.synchronize()
    comm.free()
    gpu.close()
    dist.destroy_process_group()
    return out


def leave_gpu(rank, world, port):
    """A rank leaves between steps (nothing of it in flight): it says so in the rendezvous store and aborts its own
    communicator; the others see it in the store before their next launch and abort theirs, so no collective is left
    waiting on the missing rank."""
    import time
    import torch
    import torch.distributed as dist
    sys.path.insert(0, HERE)
    from conftest import load_package
    tcu = load_package()
    from tabicl_anywhere_b200 import synth
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=60))
    torch.cuda.set_device(rank)
    gpu = tcu.Gpu(rank)
    uid = torch.zeros(tcu.COMM_ID_BYTES, dtype=torch.uint8)
    if rank == 0:
        uid = torch.frombuffer(bytearray(tcu.comm_unique_id()), dtype=torch.uint8)
    dist.broadcast(uid, 0)
    comm = tcu.Comm(gpu, bytes(uid.numpy().tobytes()), world, rank)
    cfg = synth.config("full", icl_num_blocks=2)
    wt = synth.weights(cfg, seed=51, std=0.08)
    w = tcu.GpuWeights.from_tensors(gpu, synth.icl_shape(cfg), {k: v for k, v in wt.items() if k.startswith("icl_")},
                                    for_fit=True)
    n, chunk, d = 600, 64, 512
    h = torch.from_numpy(synth.row_reps(n, d, 52)).cuda()
    y = torch.from_numpy(synth.labels(n, 10, 53)).cuda()
    torch.cuda.synchronize()
    full = tcu.fit_icl(w, h.data_ptr(), y.data_ptr(), n, chunk, 1)
    c0, nc = tcu.shard_chunks((n + chunk - 1) // chunk, world, rank)
    shard = full.slice(c0, nc)
    x = torch.from_numpy(synth.row_reps(40, d, 54)).cuda()
    o = torch.empty((40, 10), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    steps = 0
    out = {"rank": rank}
    for step in range(3):
        # before every launch: has a rank left?
        if store.check(["left"]):
            out["saw_leave_before_step"] = step
            break
        shard.stage_sharded_device(comm, x.data_ptr(), 40, 10, o.data_ptr(), stream)
        comm.wait(20000, stream)
        steps += 1
        dist.barrier()
        if step == 0 and rank == world - 1:
            # this rank leaves here: none of its work is in flight
            torch.cuda.synchronize()
            comm.abort()
            store.set("left", str(rank))
            out["left_after_step"] = step
            break
        if step == 0:
            t0 = time.time()
            while not store.check(["left"]) and time.time() - t0 < 30:
                time.sleep(0.05)
    if "left_after_step" not in out:
        comm.abort()
    out["steps"] = steps
    torch.cuda.synchronize()
    shard.free(), full.free(), w.free()
    comm.free()
    gpu.close()
    return out


if __name__ == "__main__":
    mode, rank, world, port = sys.argv[1], int(sys.argv[2]), int(sys.argv[3]), int(sys.argv[4])
    res = {"merge-cpu": merge_cpu, "push-cpu": push_cpu, "stage-gpu": stage_gpu, "leave-gpu": leave_gpu}[mode](rank, world, port)
    print(json.dumps(res), flush=True)
