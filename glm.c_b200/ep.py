"""Expert-parallel MoE prefill over ranks (one process per GPU).

The routed experts of every layer are split over the ranks of a process
group (n_routed_experts / world consecutive experts per rank); the router and
the shared expert are replicated. Per layer each rank

  1 routes its own tokens and packs one row per (token, slot) pair, grouped
    by the rank holding the pair's expert       (glm_cuda_ep_dispatch)
  2 exchanges the row counts, then the rows and their local expert ids
    (all-to-all)
  3 runs its experts on the rows it received, and the shared expert on its
    own tokens                                  (glm_cuda_ep_experts)
  4 sends every expert output back to the rank its row came from
    (all-to-all with the splits reversed)
  5 adds the shared output and the 1.8 w_k-weighted expert outputs in rank
    order                                       (glm_cuda_ep_combine)

which is apply_moe_shared_ffn_layer (infer.c:1087-1216) applied to every
token, with the expert products on the ranks that hold the experts. The
kernels are the library's (`kernels` is a GlmCuda). ExpertParallelMoE
exchanges with torch.distributed's all_to_all_single on the same stream
(NCCL on GPUs; any backend on CPU); PeerExpertParallelMoE lets the kernels
store into the other ranks' memory instead (GPUs with peer access).
"""
from __future__ import annotations

import time


class ExpertParallelMoE:
    """One rank's side of the expert-parallel MoE layers.

    kernels: a GlmCuda on which ep_setup(world, rank, max_tokens) was called
    and whose layers hold this rank's experts. dim / k_used: model sizes.
    """

    def __init__(self, kernels, dim: int, k_used: int, max_tokens: int, group=None, device=None):
        import torch
        import torch.distributed as dist

        self.torch = torch
        self.dist = dist
        self.k = kernels
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.dim = dim
        self.k_used = k_used
        self.device = device if device is not None else torch.device("cpu")
        rows = max_tokens * k_used
        f32, i32 = torch.float32, torch.int32
        self.send_rows = torch.empty(rows, dim, dtype=f32, device=self.device)
        self.send_expert = torch.empty(rows, dtype=i32, device=self.device)
        self.send_counts = torch.zeros(self.world, dtype=i32, device=self.device)
        self.recv_counts = torch.zeros(self.world, dtype=i32, device=self.device)
        cap = self.world * rows
        self.recv_rows = torch.empty(cap, dim, dtype=f32, device=self.device)
        self.recv_expert = torch.empty(cap, dtype=i32, device=self.device)
        self.out_rows = torch.empty(cap, dim, dtype=f32, device=self.device)
        self.back_rows = torch.empty(rows, dim, dtype=f32, device=self.device)
        self.last = {}

    def _stream(self):
        """The handle of torch's current stream, so that the library's kernels
        and torch's copies and collectives stay in one stream order. torch's
        default stream has handle 0, which the library would read as its own
        stream: pass cudaStreamLegacy (handle 1) for it instead."""
        if self.device.type != "cuda":
            return None
        handle = self.torch.cuda.current_stream(self.device).cuda_stream
        return handle if handle else 1

    def _a2a(self, out, inp, out_splits, in_splits):
        if self.world == 1:
            out[: inp.shape[0]].copy_(inp)
        else:
            self.dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def layer(self, layer: int, x, idx=None, w=None) -> None:
        """x [T][dim] (this rank's tokens, in place) through MoE layer `layer`."""
        T = x.shape[0]
        st = self._stream()
        self.k.ep_dispatch(layer, x, T, self.send_rows, self.send_expert, self.send_counts, stream=st)
        self._a2a(self.recv_counts, self.send_counts, None, None)
        sc = self.send_counts.tolist()   # host copy of the splits (synchronises the stream)
        rc = self.recv_counts.tolist()
        n_send, n_recv = sum(sc), sum(rc)
        self._a2a(self.recv_rows[:n_recv], self.send_rows[:n_send], rc, sc)
        self._a2a(self.recv_expert[:n_recv], self.send_expert[:n_send], rc, sc)
        self.k.ep_experts(layer, self.recv_rows, self.recv_expert, n_recv, self.out_rows, stream=st)
        self._a2a(self.back_rows[:n_send], self.out_rows[:n_recv], sc, rc)
        self.k.ep_combine(layer, x, self.back_rows, idx, w, stream=st)
        self.last = {"n_send": n_send, "n_recv": n_recv, "send_counts": sc, "recv_counts": rc}

    def layer_timed(self, layer: int, x, events: list) -> None:
        """layer() with CUDA events recorded between its phases: events[0..5]
        = before dispatch, after dispatch, after the row exchange, after the
        experts, after the exchange back, after combine."""
        T = x.shape[0]
        st = self._stream()
        events[0].record()
        self.k.ep_dispatch(layer, x, T, self.send_rows, self.send_expert, self.send_counts, stream=st)
        events[1].record()
        self._a2a(self.recv_counts, self.send_counts, None, None)
        sc = self.send_counts.tolist()
        rc = self.recv_counts.tolist()
        n_send, n_recv = sum(sc), sum(rc)
        self._a2a(self.recv_rows[:n_recv], self.send_rows[:n_send], rc, sc)
        self._a2a(self.recv_expert[:n_recv], self.send_expert[:n_send], rc, sc)
        events[2].record()
        self.k.ep_experts(layer, self.recv_rows, self.recv_expert, n_recv, self.out_rows, stream=st)
        events[3].record()
        self._a2a(self.back_rows[:n_send], self.out_rows[:n_recv], sc, rc)
        events[4].record()
        self.k.ep_combine(layer, x, self.back_rows, None, None, stream=st)
        events[5].record()
        self.last = {"n_send": n_send, "n_recv": n_recv, "send_counts": sc, "recv_counts": rc}


class PeerExpertParallelMoE:
    """The same layer with the exchange done by the library's kernels over
    peer memory (glm_cuda_ep_peer_* / glm_cuda_ep_p2p_*): the rows, the
    expert ids, the counts and the outputs travel by stores into the other
    ranks' peer regions (NVLink), with a flag per pair of ranks; no
    collective and no host round trip per layer. The process group is used
    once, to swap the regions' IPC handles.

    kernels: a GlmCuda on which ep_setup(world, rank, max_tokens) was called
    (max_tokens equal on every rank). regions: every rank's region address
    as this process sees it, to connect two library instances of one
    process directly; None swaps IPC handles over the process group.
    connect=False leaves the connection to a later connect(regions).
    """

    def __init__(self, kernels, world: int, rank: int, group=None, regions=None, connect: bool = True):
        self.k = kernels
        self.world = world
        self.rank = rank
        self.group = group
        self.region, self.handle = kernels.ep_peer_region()
        self.last = {}
        if connect:
            self.connect(regions if regions is not None else self._swap_handles())

    def _swap_handles(self) -> list[int]:
        if self.world == 1:
            return [self.region]
        import torch.distributed as dist

        handles = [None] * self.world
        dist.all_gather_object(handles, self.handle, group=self.group)
        return [self.region if r == self.rank else self.k.ep_peer_open(handles[r]) for r in range(self.world)]

    def connect(self, regions: list[int]) -> None:
        self.k.ep_peer_connect(list(regions))

    @staticmethod
    def _stream():
        import torch

        handle = torch.cuda.current_stream().cuda_stream
        return handle if handle else 1  # cudaStreamLegacy for torch's default stream

    def layer(self, layer: int, x, idx=None, w=None) -> None:
        """x [T][dim] (this rank's tokens, device, in place) through MoE layer `layer`."""
        st = self._stream()
        self.k.ep_p2p_dispatch(layer, x, x.shape[0], stream=st)
        self.k.ep_p2p_experts(layer, stream=st)
        self.k.ep_p2p_combine(layer, x, idx, w, stream=st)

    def layer_timed(self, layer: int, x, events: list) -> None:
        """layer() with CUDA events between its phases: events[0..3] = before
        dispatch, after dispatch (rows pushed), after the experts (outputs
        pushed; includes waiting for the other ranks' rows), after combine
        (includes waiting for the outputs)."""
        st = self._stream()
        events[0].record()
        self.k.ep_p2p_dispatch(layer, x, x.shape[0], stream=st)
        events[1].record()
        self.k.ep_p2p_experts(layer, stream=st)
        events[2].record()
        self.k.ep_p2p_combine(layer, x, None, None, stream=st)
        events[3].record()

    def counts(self) -> dict:
        """Rows sent to / received from every rank in the last layer (synchronises)."""
        sc, rc = self.k.ep_p2p_counts(self.world)
        self.last = {"n_send": sum(sc), "n_recv": sum(rc), "send_counts": sc, "recv_counts": rc}
        return self.last


def shard_layer(layer: dict, n_shards: int, shard: int) -> dict:
    """The arrays rank `shard` holds: router and shared expert whole, the
    routed blocks cut to experts [shard * E/n, (shard + 1) * E/n)."""
    e = layer["n_experts"] // n_shards
    out = dict(layer)
    for name in ("gate_q", "gate_s", "up_q", "up_s", "down_q", "down_s"):
        a = layer.get(name)
        out[name] = None if a is None else a[shard * e:(shard + 1) * e]
    return out
