"""Worker of test_collective: one rank of a 2-process NVLS exchange-and-Adam step, checked against
NCCL's all-reduce followed by the single-GPU Adam (to 1e-6). Prints 'unavailable' and exits 0
when the fabric has no multicast; exits 1 on a mismatch."""

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), ".."))


def main() -> int:
    rank = int(os.environ["RANK"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    import splax_b200 as sx
    from splax_b200._collective import NvlsAdam

    g0 = torch.Generator(device=dev)
    g0.manual_seed(7)  # identical parameters on every rank
    shapes = [(1001, 3), (1001, 4), (1001,)]  # 9009 floats: a ragged tail in the last shard
    lrs = [1e-2, 3e-3, 5e-2]
    init = [torch.randn(s, device=dev, generator=g0) for s in shapes]
    try:
        opt = NvlsAdam([t.clone() for t in init], lrs, dev)
    except RuntimeError as e:
        print("unavailable:", e, flush=True)
        dist.destroy_process_group()
        return 0
    ref_params = [t.clone() for t in init]
    ref = sx.Adam(ref_params, lrs)
    g = torch.Generator(device=dev)
    for it in range(3):
        g.manual_seed(100 * it + rank)  # different gradients per rank
        grads = [torch.randn(s, device=dev, generator=g) for s in shapes]
        opt.step(grads)
        summed = [t.clone() for t in grads]
        for t in summed:
            dist.all_reduce(t)
        ref.step(summed)
    torch.cuda.synchronize()
    opt.check()
    # the sums agree exactly at two ranks; the Adam arithmetic may contract differently into
    # FMAs in the two compilation units, so the parameters agree to a few ulp (1e-6 at |p| ~ 1)
    worst = max(float((a.detach() - b).abs().max()) for a, b in zip(opt.params, ref_params))
    bad = int(worst > 1e-6)
    opt.close()
    del opt
    dist.barrier()
    dist.destroy_process_group()
    # one write per rank: the ranks share the pipe, and print() writes its pieces separately
    os.write(1, f"rank {rank} mismatches {bad} max abs diff {worst}\n".encode())
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
