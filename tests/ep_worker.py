"""One rank of the two-GPU expert-parallel parity check (launched by
tests/test_ep_gpu.py through torch.distributed.run): the config-0 layer with
its experts split over the ranks, each rank's own tokens checked against the
CPU oracle (expert ids bit-exact, output within 1e-3)."""
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from __graft_entry__ import load_package
    import oracle
    from helpers import check_moe_outputs

    pkg = load_package()
    synth = pkg.synth
    L = synth.moe_layer(seed=8, zipf=1.1, **synth.CONFIG0)
    T = 96 + 37 * rank
    x = synth.tokens(800 + rank, T, 2048)
    lib = pkg.glm_cuda.GlmCuda()
    lib.init(local, 2048, 1536, 64, 4, 32, 1)
    lib.ep_setup(world, rank, 256)
    lib.upload_moe_layer(0, pkg.ep.shard_layer(L, world, rank))
    moe = pkg.ep.ExpertParallelMoE(lib, 2048, 4, 256, device=dev)
    xd = torch.from_numpy(x.copy()).to(dev)
    idx = torch.zeros((T, 4), dtype=torch.int32, device=dev)
    moe.layer(0, xd, idx)
    lib.ep_status()
    ref, ref_idx, _ = oracle.moe_layer(L, x, impl="orc")
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    worst = check_moe_outputs(x, xd.cpu().numpy(), ref, 1e-3)
    print(f"EP-OK rank {rank} worst {worst:.2e} sent {moe.last['send_counts']} recv {moe.last['recv_counts']}",
          flush=True)
    # the same layer over peer memory (IPC-mapped regions): bit-identical
    pm = pkg.ep.PeerExpertParallelMoE(lib, world, rank)
    for _ in range(2):
        xp = torch.from_numpy(x.copy()).to(dev)
        ip = torch.zeros((T, 4), dtype=torch.int32, device=dev)
        pm.layer(0, xp, ip)
        lib.ep_status()
        assert torch.equal(xp, xd) and torch.equal(ip, idx)
    last = pm.counts()
    assert last["send_counts"] == moe.last["send_counts"] and last["recv_counts"] == moe.last["recv_counts"]
    print(f"EP-P2P-OK rank {rank}", flush=True)
    dist.barrier()
    lib.free()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
