"""Expert-parallel exchange logic on CPU: world_size-2 gloo ranks run
glm_c_b200.ep.ExpertParallelMoE with stand-in kernels built from the CPU
oracle (routing, rmsnorm and the Q8 matvec of glm.c's path), so the
dispatch layout, the all-to-all splits, the return path and the rank-order
combine are checked against the oracle's whole layer without a GPU. The
stand-in implements the same contract as glm_cuda_ep_dispatch / _experts /
_combine (include/glm_cuda.h); the CUDA kernels behind those calls are
checked in tests/test_ep_gpu.py.
"""
import os
import socket

import numpy as np
import pytest

CFG = dict(dim=256, ffn=128, n_experts=8, k_used=3, gs=32)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleKernels:
    """CPU stand-in for the library's ep_* calls (test infrastructure only)."""

    def __init__(self, oracle, layer_full: dict, n_shards: int, shard: int):
        self.o = oracle
        self.L = layer_full
        self.n = n_shards
        self.shard = shard
        self.e_local = layer_full["n_experts"] // n_shards

    def _xn(self, x):
        import ctypes

        D = self.L["dim"]
        out = np.zeros_like(x)
        for t in range(x.shape[0]):
            xt = np.ascontiguousarray(x[t])
            self.o.lib("orc").orc_rmsnorm(out[t].ctypes.data, xt.ctypes.data, self.L["ffn_norm"].ctypes.data, D)
        return out

    def _ffn(self, xn_row, e):
        """SwiGLU expert e (global id; -1 = shared) on one normalised row."""
        L, gs = self.L, self.L["gs"]
        if e < 0:
            g = self.o.matvec(L["gate_sh_q"], L["gate_sh_s"], xn_row, gs)
            u = self.o.matvec(L["up_sh_q"], L["up_sh_s"], xn_row, gs)
            h = (g / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32) * u
            return self.o.matvec(L["down_sh_q"], L["down_sh_s"], h, gs)
        g = self.o.matvec(L["gate_q"][e], L["gate_s"][e], xn_row, gs)
        u = self.o.matvec(L["up_q"][e], L["up_s"][e], xn_row, gs)
        h = (g / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32) * u
        return self.o.matvec(L["down_q"][e], L["down_s"][e], h, gs)

    def ep_dispatch(self, layer, x, T, send_rows, send_expert, send_counts, stream=None):
        xh = x.numpy()[:T]
        _, idx, w = self.o.moe_layer(self.L, xh, impl="orc")
        self.xn, self.idx, self.w, self.T = self._xn(xh), idx, w, T
        K = idx.shape[1]
        self.send_pos = -np.ones((T, K), dtype=np.int64)
        pos = 0
        counts = [0] * self.n
        for d in range(self.n):
            for t in range(T):
                for k in range(K):
                    e = int(idx[t, k])
                    if e >= 0 and e // self.e_local == d:
                        send_rows[pos] = __import__("torch").from_numpy(self.xn[t])
                        send_expert[pos] = e - d * self.e_local
                        self.send_pos[t, k] = pos
                        pos += 1
                        counts[d] += 1
        for d in range(self.n):
            send_counts[d] = counts[d]

    def ep_experts(self, layer, recv_rows, recv_expert, n_recv, out_rows, stream=None):
        import torch

        for i in range(n_recv):
            e = self.shard * self.e_local + int(recv_expert[i])
            out_rows[i] = torch.from_numpy(self._ffn(recv_rows[i].numpy().copy(), e))
        self.shared = np.stack([self._ffn(self.xn[t], -1) for t in range(self.T)])

    def ep_combine(self, layer, x, back_rows, idx=None, w=None, stream=None):
        import torch

        xh = x.numpy()
        K = self.idx.shape[1]
        for t in range(self.T):
            acc = np.zeros(self.L["dim"], dtype=np.float32)
            for k in range(K):
                p = self.send_pos[t, k]
                if p < 0:
                    continue
                acc += np.float32(self.w[t, k] * np.float32(1.8)) * back_rows[p].numpy()
            xh[t] += self.shared[t] + acc


def _rank(rank, world, port, result_q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package

        pkg = load_package()
        import oracle

        L = pkg.synth.moe_layer(seed=77, zipf=1.1, **CFG)
        T = 5 + 3 * rank  # ragged: the ranks route different numbers of tokens
        x = pkg.synth.tokens(700 + rank, T, CFG["dim"])
        ref, ref_idx, _ = oracle.moe_layer(L, x, impl="orc")
        k = OracleKernels(oracle, L, world, rank)
        moe = pkg.ep.ExpertParallelMoE(k, CFG["dim"], CFG["k_used"], max_tokens=16)
        xt = torch.from_numpy(x.copy())
        moe.layer(0, xt)
        err = float(np.abs(xt.numpy() - ref).max() / np.abs(ref - x).max())
        result_q.put((rank, err, moe.last))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_ep_exchange_ranks_match_oracle(world):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, err, last in res:
        # the stand-in's SiLU runs in float64: last-bit differences from
        # glm.c's expf, magnified where the FFN output nearly cancels; a
        # misrouted row or a wrong split gives errors of order 1
        assert err < 1e-4, f"rank {rank}: relative max error {err}"
        assert sum(last["send_counts"]) == (5 + 3 * rank) * CFG["k_used"]
    # what rank a sent to rank b is what rank b received from rank a
    for a in range(world):
        for b in range(world):
            assert res[a][2]["send_counts"][b] == res[b][2]["recv_counts"][a]


def test_shard_layer_cuts_routed_blocks(pkg):
    L = pkg.synth.moe_layer(seed=3, **CFG)
    s = pkg.ep.shard_layer(L, 4, 2)
    assert s["gate_q"].shape[0] == 2 and np.array_equal(s["gate_q"], L["gate_q"][4:6])
    assert s["router"] is L["router"] and s["down_sh_q"] is L["down_sh_q"]


class _FakePeerKernels:
    """Records what PeerExpertParallelMoE asks of the library's peer calls
    (test infrastructure only): region addresses and IPC handles are made up
    from the rank, opening a handle maps it to a distinct made-up address."""

    def __init__(self, rank):
        self.rank = rank
        self.opened = []
        self.connected = None

    def ep_peer_region(self):
        return 0x10000000 * (self.rank + 1), bytes([self.rank + 1]) * 64

    def ep_peer_open(self, handle):
        self.opened.append(handle)
        return 0x70000000 + 0x100000 * handle[0]

    def ep_peer_connect(self, regions):
        self.connected = list(regions)


def _peer_rank(rank, world, port, result_q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from __graft_entry__ import load_package

        pkg = load_package()
        k = _FakePeerKernels(rank)
        pkg.ep.PeerExpertParallelMoE(k, world, rank)
        result_q.put((rank, k.connected, [h[0] for h in k.opened]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_regions_swap_handles_over_the_group(world):
    """Every rank connects to `world` regions in rank order: its own region
    at its own index, every other rank's opened from that rank's handle."""
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_peer_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    res = sorted(q.get(timeout=5) for _ in range(world))
    for rank, connected, opened in res:
        assert len(connected) == world
        for r in range(world):
            want = 0x10000000 * (rank + 1) if r == rank else 0x70000000 + 0x100000 * (r + 1)
            assert connected[r] == want
        assert sorted(opened) == [r + 1 for r in range(world) if r != rank]
