"""Worker of tests/test_dist_gpu.py: one rank of the distributed single-signal
convolution over NCCL.  Launched by torchrun; rank 0 saves the gathered
result.  usage: dist_gpu_worker.py <n> <out.npy> [nccl|p2p]"""
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    n, out = int(sys.argv[1]), sys.argv[2]
    mode = sys.argv[3] if len(sys.argv) > 3 else "nccl"
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60))
    try:
        from fufft_b200 import ops
        from fufft_b200.distributed import (GpuBackend, PeerBlocks, conv_distributed, conv_distributed_p2p,
                                            filter_block, gather_signal, scatter_signal)
        from oracle.oracle import Oracle
        ops.init()
        rank, world = dist.get_rank(), dist.get_world_size()
        be = GpuBackend()
        plan = be.plan(n, world)
        rng = np.random.default_rng(n + world)
        a = (rng.standard_normal(n) + 1j * rng.standard_normal(n)).astype(np.complex64)
        spec = (np.fft.fft(rng.uniform(-1, 1, n) + 1j * rng.uniform(-1, 1, n)) / n).astype(np.complex64)
        rev = Oracle().rev_table(plan.chain, n)
        b_chain = torch.from_numpy(np.ascontiguousarray(spec[rev])).cuda()
        x = scatter_signal(torch.from_numpy(a).cuda(), n, world, rank)
        if mode == "p2p":
            peers = PeerBlocks(plan.n_blk)
            for _ in range(2):     # the buffers are reused by consecutive calls
                x = scatter_signal(torch.from_numpy(a).cuda(), n, world, rank)
                y = conv_distributed_p2p(x, filter_block(b_chain, n, world, rank), n, peers, backend=be, plan=plan)
        else:
            y = conv_distributed(x, filter_block(b_chain, n, world, rank), n, backend=be, plan=plan)
        parts = [torch.empty_like(torch.view_as_real(y)) for _ in range(world)]
        dist.all_gather(parts, torch.view_as_real(y))
        torch.cuda.synchronize()
        if mode == "p2p":
            peers.close()
        if rank == 0:
            full = gather_signal([torch.view_as_complex(p) for p in parts], n).cpu().numpy()
            np.save(out, full)
            np.save(out + ".plan.npy", np.array([plan.one_kernel, plan.r_out, plan.mid, *plan.chain]))
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
