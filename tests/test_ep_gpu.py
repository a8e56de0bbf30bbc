"""Expert-parallel prefill on the GPU through the C-ABI (glm_cuda_ep_*):
expert ids bit-identical to glm.c's CPU path, MoE-layer outputs within 1e-3
relative L2, for one shard, for two shards emulated in one
process (two copies of the library, one per shard, exchanging through device
copies) and, where two GPUs are present, for two ranks over NCCL.
"""
import ctypes
import os
import shutil
import subprocess
import sys

import numpy as np
import pytest

from helpers import check_moe_outputs

pytestmark = pytest.mark.gpu

TOL = 1e-3
LEGACY = 1  # cudaStreamLegacy: the library's kernels in order with torch's default-stream copies
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def torch_cuda():
    torch = pytest.importorskip("torch")
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch


def _lib_copy(pkg, tmp_path, name):
    """A second, independent instance of the library (its own global state)."""
    gc = pkg.glm_cuda
    path = str(tmp_path / name)
    shutil.copy(gc.LIB_PATH, path)
    L = ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL)
    gc._signatures(L)
    obj = gc.GlmCuda.__new__(gc.GlmCuda)
    obj.L = L
    return obj


def test_ep_one_shard_matches_oracle(torch_cuda, pkg, oracle_mod):
    torch = torch_cuda
    synth = pkg.synth
    L = synth.moe_layer(seed=5, zipf=1.1, **synth.CONFIG0)
    T = 256
    x = synth.tokens(505, T, 2048)
    lib = pkg.glm_cuda.GlmCuda()
    lib.init(0, 2048, 1536, 64, 4, 32, 1)
    lib.ep_setup(1, 0, T)
    lib.upload_moe_layer(0, L)
    moe = pkg.ep.ExpertParallelMoE(lib, 2048, 4, T, device=torch.device("cuda", 0))
    xd = torch.from_numpy(x.copy()).cuda()
    idx = torch.zeros((T, 4), dtype=torch.int32, device="cuda")
    w = torch.zeros((T, 4), dtype=torch.float32, device="cuda")
    moe.layer(0, xd, idx, w)
    lib.ep_status()
    ref, ref_idx, ref_w = oracle_mod.moe_layer(L, x, impl="orc")
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    np.testing.assert_allclose(w.cpu().numpy(), ref_w, rtol=0, atol=1e-4)
    worst = check_moe_outputs(x, xd.cpu().numpy(), ref, TOL)
    assert moe.last["n_recv"] == T * 4
    print(f"ep 1 shard: worst rel L2 {worst:.2e}")
    lib.free()


@pytest.mark.parametrize("cfg,T", [(dict(dim=512, ffn=256, n_experts=16, k_used=4, gs=32), (40, 23)),
                                   (dict(dim=2048, ffn=1536, n_experts=64, k_used=4, gs=32), (200, 131))])
def test_ep_two_shards_one_gpu(cfg, T, torch_cuda, pkg, oracle_mod, tmp_path):
    """Shards 0 and 1 as two library instances on one GPU; the all-to-all is
    done with device copies in the order the ranks would exchange."""
    torch = torch_cuda
    synth, ep = pkg.synth, pkg.ep
    L = synth.moe_layer(seed=6, zipf=1.1, **cfg)
    D, K = cfg["dim"], cfg["k_used"]
    xs = [synth.tokens(600 + r, T[r], D) for r in range(2)]
    libs = [_lib_copy(pkg, tmp_path, f"libglm_shard{r}.so") for r in range(2)]
    bufs = []
    for r, lib in enumerate(libs):
        lib.init(0, D, cfg["ffn"], cfg["n_experts"], K, 32, 1)
        lib.ep_setup(2, r, max(T))
        lib.upload_moe_layer(0, ep.shard_layer(L, 2, r))
        rows = max(T) * K
        bufs.append(dict(x=torch.from_numpy(xs[r].copy()).cuda(),
                         send=torch.zeros(rows, D, device="cuda"),
                         sexp=torch.zeros(rows, dtype=torch.int32, device="cuda"),
                         cnt=torch.zeros(2, dtype=torch.int32, device="cuda"),
                         idx=torch.zeros(T[r], K, dtype=torch.int32, device="cuda")))
    for r, lib in enumerate(libs):
        b = bufs[r]
        lib.ep_dispatch(0, b["x"], T[r], b["send"], b["sexp"], b["cnt"], stream=LEGACY)
    torch.cuda.synchronize()
    cnt = [b["cnt"].tolist() for b in bufs]
    off = [[0, cnt[r][0]] for r in range(2)]
    outs = []
    for d, lib in enumerate(libs):  # rank d receives from ranks 0, 1 in order
        rows = torch.cat([bufs[s]["send"][off[s][d]:off[s][d] + cnt[s][d]] for s in range(2)])
        exps = torch.cat([bufs[s]["sexp"][off[s][d]:off[s][d] + cnt[s][d]] for s in range(2)])
        out = torch.zeros_like(rows)
        lib.ep_experts(0, rows, exps, rows.shape[0], out, stream=LEGACY)
        torch.cuda.synchronize()
        outs.append(out)
    for s, lib in enumerate(libs):  # back to the senders, in their send order
        parts = []
        for d in range(2):
            start = sum(cnt[q][d] for q in range(s))
            parts.append(outs[d][start:start + cnt[s][d]])
        back = torch.cat(parts)
        lib.ep_combine(0, bufs[s]["x"], back, bufs[s]["idx"], stream=LEGACY)
        lib.ep_status()
    for r in range(2):
        ref, ref_idx, _ = oracle_mod.moe_layer(L, xs[r], impl="orc")
        np.testing.assert_array_equal(bufs[r]["idx"].cpu().numpy(), ref_idx)
        worst = check_moe_outputs(xs[r], bufs[r]["x"].cpu().numpy(), ref, TOL)
        print(f"ep 2 shards rank {r}: worst rel L2 {worst:.2e}")
    for lib in libs:
        lib.free()


def test_ep_p2p_one_shard_matches_alltoall_path(torch_cuda, pkg, oracle_mod):
    """The peer-memory exchange (one shard: the rank pushes into its own
    region) gives bit-identical outputs, ids and weights to the all-to-all
    path, over several layer calls (the flags' epochs advance)."""
    torch = torch_cuda
    synth = pkg.synth
    L = synth.moe_layer(seed=5, zipf=1.1, **synth.CONFIG0)
    T = 256
    x = synth.tokens(505, T, 2048)
    lib = pkg.glm_cuda.GlmCuda()
    lib.init(0, 2048, 1536, 64, 4, 32, 1)
    lib.ep_setup(1, 0, T)
    lib.upload_moe_layer(0, L)
    dev = torch.device("cuda", 0)
    a2a = pkg.ep.ExpertParallelMoE(lib, 2048, 4, T, device=dev)
    xa = torch.from_numpy(x.copy()).cuda()
    ia = torch.zeros((T, 4), dtype=torch.int32, device=dev)
    wa = torch.zeros((T, 4), dtype=torch.float32, device=dev)
    a2a.layer(0, xa, ia, wa)
    p2p = pkg.ep.PeerExpertParallelMoE(lib, 1, 0)
    for _ in range(3):
        xp = torch.from_numpy(x.copy()).cuda()
        ip = torch.zeros((T, 4), dtype=torch.int32, device=dev)
        wp = torch.zeros((T, 4), dtype=torch.float32, device=dev)
        p2p.layer(0, xp, ip, wp)
        lib.ep_status()
        assert torch.equal(xp, xa) and torch.equal(ip, ia) and torch.equal(wp, wa)
    last = p2p.counts()
    assert last["send_counts"] == [T * 4] and last["recv_counts"] == [T * 4]
    ref, ref_idx, _ = oracle_mod.moe_layer(L, x, impl="orc")
    np.testing.assert_array_equal(ip.cpu().numpy(), ref_idx)
    worst = check_moe_outputs(x, xp.cpu().numpy(), ref, TOL)
    print(f"ep p2p 1 shard: worst rel L2 {worst:.2e}")
    lib.free()


SMALL = dict(dim=512, ffn=256, n_experts=16, k_used=4, gs=32)


@pytest.mark.parametrize("cfg,T", [(SMALL, (40, 23)), (SMALL, (17, 40, 1, 33)),
                                   (SMALL, (9, 30, 2, 41, 16, 5, 28, 12)),
                                   (dict(dim=2048, ffn=1536, n_experts=64, k_used=4, gs=32), (200, 131))])
def test_ep_p2p_shards_one_gpu(cfg, T, torch_cuda, pkg, oracle_mod, tmp_path):
    """n = len(T) shards as n library instances on one GPU, connected through
    each other's peer regions: each phase is issued for every shard before
    the next phase, in one stream, so every wait is already satisfied when
    it runs. Two layer calls (epochs 1 and 2). With 8 shards of 16 experts a
    rank holds 2 experts, fewer than the 4 a token picks (a token sends at
    most 2 rows to one rank); one rank routes a single token."""
    torch = torch_cuda
    synth, ep = pkg.synth, pkg.ep
    n = len(T)
    L = synth.moe_layer(seed=6, zipf=1.1, **cfg)
    D, K = cfg["dim"], cfg["k_used"]
    xs = [synth.tokens(600 + r, T[r], D) for r in range(n)]
    libs = [_lib_copy(pkg, tmp_path, f"libglm_p2p{r}.so") for r in range(n)]
    for r, lib in enumerate(libs):
        lib.init(0, D, cfg["ffn"], cfg["n_experts"], K, 32, 1)
        lib.ep_setup(n, r, max(T))
        lib.upload_moe_layer(0, ep.shard_layer(L, n, r))
    pms = [ep.PeerExpertParallelMoE(lib, n, r, connect=False) for r, lib in enumerate(libs)]
    regions = [pm.region for pm in pms]
    for pm in pms:
        pm.connect(regions)
    for rep in range(2):
        xd = [torch.from_numpy(xs[r].copy()).cuda() for r in range(n)]
        idx = [torch.zeros(T[r], K, dtype=torch.int32, device="cuda") for r in range(n)]
        for r, lib in enumerate(libs):
            lib.ep_p2p_dispatch(0, xd[r], T[r], stream=LEGACY)
        for r, lib in enumerate(libs):
            lib.ep_p2p_experts(0, stream=LEGACY)
        for r, lib in enumerate(libs):
            lib.ep_p2p_combine(0, xd[r], idx[r], None, stream=LEGACY)
        for lib in libs:
            lib.ep_status()
        for r in range(n):
            ref, ref_idx, _ = oracle_mod.moe_layer(L, xs[r], impl="orc")
            np.testing.assert_array_equal(idx[r].cpu().numpy(), ref_idx)
            worst = check_moe_outputs(xs[r], xd[r].cpu().numpy(), ref, TOL)
            print(f"ep p2p {n} shards call {rep} rank {r}: worst rel L2 {worst:.2e}")
    c = [pm.counts() for pm in pms]
    for a in range(n):
        assert sum(c[a]["send_counts"]) == T[a] * K
        for b in range(n):
            assert c[a]["send_counts"][b] == c[b]["recv_counts"][a]
    for lib in libs:
        lib.free()


def test_ep_p2p_connect_refuses_mismatched_regions(torch_cuda, pkg, tmp_path):
    """A region laid out for another max_tokens is refused at connect (the
    kernels' stores into it would otherwise land outside it)."""
    import glm_c_b200.glm_cuda as gc

    libs = [_lib_copy(pkg, tmp_path, f"libglm_mis{r}.so") for r in range(2)]
    for r, lib in enumerate(libs):
        lib.init(0, 512, 256, 16, 4, 32, 1)
        lib.ep_setup(2, r, 32 if r == 0 else 48)
    pms = [pkg.ep.PeerExpertParallelMoE(lib, 2, r, connect=False) for r, lib in enumerate(libs)]
    regions = [pm.region for pm in pms]
    for pm in pms:
        with pytest.raises(gc.GlmCudaError):
            pm.connect(regions)
    with pytest.raises(gc.GlmCudaError):  # not connected: the layer calls refuse too
        libs[0].ep_p2p_experts(0, stream=LEGACY)
    for lib in libs:
        lib.free()


def test_ep_single_rank_calls_refuse_sharded_layers(torch_cuda, pkg):
    import glm_c_b200.glm_cuda as gc

    lib = pkg.glm_cuda.GlmCuda()
    cfg = dict(dim=256, ffn=128, n_experts=8, k_used=2, gs=32)
    lib.init(0, 256, 128, 8, 2, 32, 1)
    lib.ep_setup(2, 1, 4)
    lib.upload_moe_layer(0, pkg.ep.shard_layer(pkg.synth.moe_layer(seed=1, **cfg), 2, 1))
    with pytest.raises(gc.GlmCudaError):
        lib.moe_layer(0, np.zeros((1, 256), np.float32), 2)
    lib.free()


def test_ep_two_ranks_nccl(torch_cuda):
    """Two ranks, one GPU each: the NCCL all-to-all exchange, then the
    peer-memory exchange through IPC-mapped regions, bit-identical to it
    (skipped with fewer GPUs)."""
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29621", os.path.join(ROOT, "tests", "ep_worker.py")]
    r = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, cwd=ROOT)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("EP-OK") == 2, r.stdout[-3000:]
    assert r.stdout.count("EP-P2P-OK") == 2, r.stdout[-3000:]
