"""Multi-rank host logic on CPU (gloo, world_size 2).

The multi-GPU step splits the cameras over ranks and sums the gaussian gradients with one
all-reduce. These tests run that decomposition with the oracle standing in for each rank's
GPU render: the all-reduced shard gradients must equal the single-process gradient of the full
camera batch, and a rank that leaves before the collective must make the other rank's
all-reduce fail after a short timeout instead of hanging.
"""

from __future__ import annotations

import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scene():
    sys.path.insert(0, str(ROOT / "tests"))
    sys.path.insert(0, str(ROOT))
    from conftest import random_scene, viewmat

    n, H, W, B = 300, 48, 48, 4
    m, s, q, c, op, bg = random_scene(n, 4)
    views = np.stack([viewmat(0.1 * i, -0.1, 5.0 - 0.2 * i) for i in range(B)])
    target = np.random.default_rng(2).uniform(size=(B, H, W, 3)).astype(np.float32)
    return (m, s, q, c, op, bg), views, target, (n, H, W, B)


def _grads_for(cams, scene, views, target, dims):
    import _oracle_chain as ch

    (m, s, q, c, op, bg), (n, H, W, B) = scene, dims
    cam = {"img_shape": (H, W), "f": (float(H), float(H)), "c": (W // 2, H // 2)}
    total = [np.zeros_like(x, dtype=np.float64) for x in (m, s, q, c, op)]
    for b in cams:
        img, _, _ = ch.render(m, s, q, c, op, bg, views[b], **cam)
        v_img = (2.0 * (img - target[b]) / (B * H * W * 3)).astype(np.float32)
        g = ch.grads(m, s, q, c, op, bg, views[b], v_img, **cam)
        for k in range(5):
            total[k] += g[k]
    return np.concatenate([t.reshape(-1) for t in total])


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=timedelta(seconds=20))
    scene, views, target, dims = _scene()
    B = dims[3]
    per = B // world
    flat = torch.tensor(_grads_for(range(rank * per, (rank + 1) * per), scene, views, target, dims))
    dist.all_reduce(flat)
    if rank == 0:
        np.save(Path(out_dir) / "reduced.npy", flat.numpy())
    dist.destroy_process_group()


def test_sharded_gradients_sum_to_full_gradient(tmp_path, oracle_lib):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    reduced = np.load(tmp_path / "reduced.npy")
    scene, views, target, dims = _scene()
    full = _grads_for(range(dims[3]), scene, views, target, dims)
    assert np.allclose(reduced, full, rtol=1e-9, atol=1e-12)


def _leaver(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    if rank == 1:
        return  # leaves between steps, without joining the next collective
    try:
        dist.all_reduce(torch.ones(4))
        outcome = "completed"
    except Exception as e:  # noqa: BLE001
        outcome = f"error: {type(e).__name__}"
    (Path(out_dir) / "outcome.txt").write_text(outcome)


def test_missing_rank_fails_the_collective(tmp_path):
    port = _free_port()
    ctx = mp.start_processes(_leaver, args=(2, port, str(tmp_path)), nprocs=2, join=False,
                             start_method="spawn")
    while not ctx.join(timeout=60):
        pass
    outcome = (tmp_path / "outcome.txt").read_text()
    assert outcome.startswith("error"), outcome


def _split_worker(rank, world, port, out_dir):
    """bench.py's SplitAllReduce on CPU tensors: the hook-started all-reduce of params 3 and 4
    and the closing one of the rest and the loss must give the summed gradients and loss."""
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    from bench import SplitAllReduce

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    shapes = [(7, 3), (7, 3), (7, 4), (7, 3), (7,)]
    params = [torch.zeros(s, dtype=torch.float64, requires_grad=True) for s in shapes]
    split = SplitAllReduce(params, early=(3, 4))
    results = []
    for step in range(2):  # two steps: the hooks re-arm
        for p in params:
            p.grad = None
        g = torch.Generator().manual_seed(100 * rank + step)
        w = [torch.randn(s, generator=g, dtype=torch.float64) for s in shapes]
        loss = sum((p * wk).sum() for p, wk in zip(params, w)) + float(rank + 1)
        split.arm()
        loss.backward()
        total = split.finish(loss)
        results.append([p.grad.clone() for p in params] + [total.detach().reshape(1)])
    torch.save(results, Path(out_dir) / f"split_{rank}.pt")
    dist.destroy_process_group()


def test_split_all_reduce_sums_gradients_and_loss(tmp_path):
    import torch

    port = _free_port()
    mp.start_processes(_split_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    r0 = torch.load(tmp_path / "split_0.pt")
    r1 = torch.load(tmp_path / "split_1.pt")
    shapes = [(7, 3), (7, 3), (7, 4), (7, 3), (7,)]
    for step in range(2):
        exp = [torch.zeros(s, dtype=torch.float64) for s in shapes]
        for rank in range(2):
            g = torch.Generator().manual_seed(100 * rank + step)
            w = [torch.randn(s, generator=g, dtype=torch.float64) for s in shapes]
            for k in range(5):
                exp[k] += w[k]
        for k in range(5):
            assert torch.allclose(r0[step][k], exp[k]) and torch.equal(r0[step][k], r1[step][k])
        assert float(r0[step][5]) == float(r1[step][5])
