"""splax_project_noalloc: the projection for callers that cannot allocate device memory.

Some callers of this library must not let it call cudaMalloc -- an XLA custom call inside a
JAX process whose allocator has already reserved most of the GPU, or an embedder with a fixed
device-memory budget. For them the projection has a second entry point whose scan scratch is a
fixed 128 KiB + 16 byte array compiled into the library (at most 16,777,216 camera-gaussian
pairs per call). This test calls it through the C ABI twice in a row, before the library's
allocating projection has run in this test, so its first call does the per-device set-up, and
requires the same outputs, bit for bit, as splax_project -- the tolerance of every other
projection test -- so a stale array left by the first call would show up in the second. The
device's free memory must not change across the second call. After one eager call, a call
also records into a CUDA graph under global capture mode, and the replay gives the same
outputs. It also checks that an oversized call is refused with a clear message.

The file is named to be collected last, so a run that stops at the first failure has already
run every other test; it passes alone in a fresh process as well as after the others.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import cam, random_scene, viewmat

pytestmark = pytest.mark.gpu


def _call(lib, fn, ins, n, H, W, total, seed_fill):
    from splax_b200 import _lib

    m, s, q, vm, op, tf, ids = ins
    dev = m.device
    outs = [torch.full((total, 2), seed_fill, device=dev), torch.full((total,), seed_fill, device=dev),
            torch.full((total,), -7, device=dev, dtype=torch.int32),
            torch.full((total, 3), seed_fill, device=dev),
            torch.full((total,), -7, device=dev, dtype=torch.int32),
            torch.full((total,), -7, device=dev, dtype=torch.int32)]
    p = _lib.ptr
    c = cam(H, W)
    rc = getattr(lib, fn)(
        p(m), m.numel() // 3, p(s), s.numel() // 3, p(q), q.numel() // 4, p(vm), vm.numel() // 4,
        p(op), op.numel(), p(tf), tf.numel() // 16, p(ids), n, 1, 0, H, W, c["f"][0], c["f"][1],
        float(c["c"][0]), float(c["c"][1]), 1.0, 0.01, total, *[p(o) for o in outs],
        _lib.stream_of(m))
    _lib.check(rc)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in outs]


def test_project_noalloc_matches_project():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from splax_b200 import _lib

    lib = _lib.load()
    n, H, W = 40_000, 240, 320
    m, s, q, c, op, bg = random_scene(n, 21, spread=1.0, smin=0.005, smax=0.05)
    views = np.stack([viewmat(0.0), viewmat(0.25), viewmat(-0.3, 0.1, 4.5)])
    B = views.shape[0]
    t = lambda a: torch.tensor(np.ascontiguousarray(a), device="cuda")  # noqa: E731
    ins = (t(m), t(s), t(np.roll(q, -1, -1)), t(views.reshape(-1, 4)), t(op),
           torch.zeros((1, 4, 4), device="cuda"), torch.full((1,), -1, device="cuda",
                                                              dtype=torch.int32))
    # two calls in a row over differently stale buffers; the first one sets the device up
    got = [_call(lib, "splax_project_noalloc", ins, n, H, W, B * n, fill)
           for fill in (3.0, -5.0)]
    ref = _call(lib, "splax_project", ins, n, H, W, B * n, 0.0)
    assert ref[5][-1] > 0  # the scene hits tiles
    for k in range(2):
        for name, a, b in zip(["xys", "depths", "radii", "conics", "num_tiles_hit", "cum"],
                              got[k], ref):
            assert np.array_equal(a, b), f"call {k}: {name} differs"
    # a single-camera call after the batched ones must not see the batched call's scan words
    got1 = _call(lib, "splax_project_noalloc", (ins[0], ins[1], ins[2], t(viewmat()), ins[4],
                                                 ins[5], ins[6]), n, H, W, n, 1.0)
    ref1 = _call(lib, "splax_project", (ins[0], ins[1], ins[2], t(viewmat()), ins[4], ins[5],
                                        ins[6]), n, H, W, n, 0.0)
    for a, b in zip(got1, ref1):
        assert np.array_equal(a, b)


def test_project_noalloc_leaves_free_memory_unchanged():
    """Once set up, a call changes nothing in the device's free memory."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from splax_b200 import _lib

    lib = _lib.load()
    n, H, W = 20_000, 200, 300
    m, s, q, c, op, bg = random_scene(n, 23, spread=1.0, smin=0.005, smax=0.05)
    t = lambda a: torch.tensor(np.ascontiguousarray(a), device="cuda")  # noqa: E731
    ins = (t(m), t(s), t(np.roll(q, -1, -1)), t(viewmat()), t(op),
           torch.zeros((1, 4, 4), device="cuda"), torch.full((1,), -1, device="cuda",
                                                              dtype=torch.int32))
    outs = [torch.empty((n, 2), device="cuda"), torch.empty((n,), device="cuda"),
            torch.empty((n,), device="cuda", dtype=torch.int32), torch.empty((n, 3), device="cuda"),
            torch.empty((n,), device="cuda", dtype=torch.int32),
            torch.empty((n,), device="cuda", dtype=torch.int32)]
    p = _lib.ptr
    cm = cam(H, W)

    def call():
        _lib.check(lib.splax_project_noalloc(
            p(ins[0]), n, p(ins[1]), n, p(ins[2]), n, p(ins[3]), 4, p(ins[4]), n, p(ins[5]), 1,
            p(ins[6]), n, 1, 0, H, W, cm["f"][0], cm["f"][1], float(cm["c"][0]),
            float(cm["c"][1]), 1.0, 0.01, n, *[p(o) for o in outs], _lib.stream_of(ins[0])))
        torch.cuda.synchronize()

    call()  # set-up (module load, symbol address) happens here at the latest
    free0, _ = torch.cuda.mem_get_info()
    call()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_project_noalloc_records_into_a_cuda_graph():
    """After one eager call, a call records into a CUDA graph under global capture mode (which
    refuses cudaMalloc and every other unsafe call while the capture runs); replayed over
    overwritten outputs, the graph gives splax_project's outputs bit for bit."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from splax_b200 import _lib

    lib = _lib.load()
    n, H, W = 30_000, 224, 288
    m, s, q, c, op, bg = random_scene(n, 25, spread=1.0, smin=0.005, smax=0.05)
    views = np.stack([viewmat(0.1), viewmat(-0.2, 0.05, 4.8)])
    B = views.shape[0]
    t = lambda a: torch.tensor(np.ascontiguousarray(a), device="cuda")  # noqa: E731
    ins = (t(m), t(s), t(np.roll(q, -1, -1)), t(views.reshape(-1, 4)), t(op),
           torch.zeros((1, 4, 4), device="cuda"), torch.full((1,), -1, device="cuda",
                                                              dtype=torch.int32))
    total = B * n
    outs = [torch.empty((total, 2), device="cuda"), torch.empty((total,), device="cuda"),
            torch.empty((total,), device="cuda", dtype=torch.int32),
            torch.empty((total, 3), device="cuda"),
            torch.empty((total,), device="cuda", dtype=torch.int32),
            torch.empty((total,), device="cuda", dtype=torch.int32)]
    p = _lib.ptr
    cm = cam(H, W)

    def call():
        return lib.splax_project_noalloc(
            p(ins[0]), n, p(ins[1]), n, p(ins[2]), n, p(ins[3]), 4 * B, p(ins[4]), n, p(ins[5]),
            1, p(ins[6]), n, 1, 0, H, W, cm["f"][0], cm["f"][1], float(cm["c"][0]),
            float(cm["c"][1]), 1.0, 0.01, total, *[p(o) for o in outs], _lib.stream_of(ins[0]))

    _lib.check(call())  # the per-device set-up happens outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, capture_error_mode="global"):
        rc = call()
    _lib.check(rc)
    for o in outs:
        o.fill_(-9)
    graph.replay()
    torch.cuda.synchronize()
    got = [o.cpu().numpy() for o in outs]
    ref = _call(lib, "splax_project", ins, n, H, W, total, 0.0)
    assert ref[5][-1] > 0
    for name, a, b in zip(["xys", "depths", "radii", "conics", "num_tiles_hit", "cum"], got, ref):
        assert np.array_equal(a, b), f"{name} differs after the graph replay"
    del graph


def test_project_noalloc_rejects_oversized_calls():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from splax_b200 import _lib

    lib = _lib.load()
    n = 1 << 22
    total = 5 * n  # 20,971,520 pairs > 16,777,216
    dummy = torch.zeros(16, device="cuda")
    p = _lib.ptr
    rc = lib.splax_project_noalloc(
        p(dummy), n, p(dummy), n, p(dummy), n, p(dummy), 4 * 5, p(dummy), n, p(dummy), 1,
        p(dummy), n, 1, 0, 64, 64, 64.0, 64.0, 32.0, 32.0, 1.0, 0.01, total, p(dummy), p(dummy),
        p(dummy), p(dummy), p(dummy), p(dummy), _lib.stream_of(dummy))
    assert rc == _lib.SPLAX_ERR_INVALID_ARGUMENT
    assert "static scratch limit" in lib.splax_last_error().decode()
