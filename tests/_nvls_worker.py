"""Worker of test_collective: one rank of a 2-process NVLS gradient all-reduce, checked against
NCCL's all-reduce of the same arrays. Prints 'unavailable' and exits 0 when the fabric has no
multicast; exits 1 on a mismatch."""

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
    from splax_b200._collective import GradAllReduce

    n = 12_347  # a ragged tail (n % 4 != 0) in the last rank's shard
    shapes = [(n, 3), (n, 4), (n,), (1,)]
    try:
        red = GradAllReduce(shapes, dev)
    except RuntimeError as e:
        print("unavailable:", e, flush=True)
        dist.destroy_process_group()
        return 0
    bad = 0
    g = torch.Generator(device=dev)
    for it in range(3):  # the epochs advance; results stay exact
        g.manual_seed(1000 * it + rank)
        ts = [torch.randn(s, device=dev, generator=g) for s in shapes]
        ref = [t.clone() for t in ts]
        for t in ref:
            dist.all_reduce(t)
        out = red.reduce(ts)
        torch.cuda.synchronize()
        bad += sum(int(not torch.equal(a, b)) for a, b in zip(out, ref))
    red.check()
    red.close()
    del red
    dist.barrier()
    dist.destroy_process_group()
    # one write per rank: the ranks share the pipe, and print() writes its pieces separately
    os.write(1, f"rank {rank} mismatches {bad}\n".encode())
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
