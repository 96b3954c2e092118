"""Expert-parallel MoE MLP across ranks (one process per GPU).

Rank r owns experts [r * E / W, (r + 1) * E / W). One forward:

  1. dispatch plan: stable sort of this rank's T*k slots by expert
     (moe_align with block_m = 1); the sorted order is also sorted by owning
     rank, so rows bound for rank d form one contiguous run
  2. counts exchange: per-(source, local expert) slot counts, all_to_all
  3. token dispatch: gather x rows in sorted order, all_to_all_single over
     NCCL (NVLink / NVSwitch)
  4. local experts: the received rows (grouped by source, then by expert)
     run through the fused expert MLP with k = 1 and unit weights
  5. return: expert outputs travel back with the inverse all_to_all_single
  6. combine: y[t] = sum_j topk_weights[t, j] * out[slot_pos[t * k + j]]
     (deterministic fp32 sum, moe_combine_rows)

The reference has no distributed code; this layer is what the multi-GPU
workloads need around the single-GPU hot path. The device work of steps 1, 3,
4 and 6 goes through `ops` (CudaOps = libmoe_b200 kernels); the collectives
are torch.distributed calls, so the exchange logic also runs with the gloo
backend on CPU tensors when `ops` is replaced (the CPU tests do that).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib
from . import moe as _moe


class CudaOps:
    """Device work of the EP layer on libmoe_b200."""

    def sort_slots(self, topk_ids: torch.Tensor, num_experts: int):
        a = _moe.moe_align(topk_ids, num_experts, block_m=1)
        return a["sorted_slots"], a["slot_pos"], a["group_sizes"], a["tile_table"][1:2]

    def gather(self, x: torch.Tensor, sorted_slots: torch.Tensor, top_k: int, rows: int,
               rows_dev: torch.Tensor | None = None) -> torch.Tensor:
        return _moe.gather_rows(x, sorted_slots, top_k, rows, rows_dev=rows_dev)

    def expert_forward(self, x_rows, local_ids, w13, w2, scales):
        return _moe.fused_expert_rows(x_rows, w13, w2, local_ids, scales=scales)

    def combine(self, o_back, slot_pos, topk_weights, out_dtype):
        T, k = topk_weights.shape
        H = o_back.shape[1]
        y = torch.empty((T, H), dtype=out_dtype, device=o_back.device)
        if T == 0:
            return y
        if o_back.shape[0] == 0:  # every slot dropped
            return y.zero_()
        _lib.call("moe_combine_rows", o_back.data_ptr(), _moe._code(o_back), H, slot_pos.data_ptr(),
                  topk_weights.data_ptr(), T, k, y.data_ptr(), _moe._code(y), _moe._stream(o_back.device))
        return y


class ExpertParallelMoE:
    """MoE expert MLP with experts sharded over the ranks of `group`.

    w13 / w2: this rank's experts in the reference's logical layout
    ([E_local, H, 2I] / [E_local, I, H], K-major storage), or int8 with
    scales=(w13_scale [E_local, 2I], w2_scale [E_local, H]).
    Call: layer(x [T, H], topk_weights [T, k], topk_ids [T, k] global ids).
    """

    def __init__(self, w13, w2, num_experts: int, scales=None, group=None, ops=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError("num_experts must be divisible by the world size")
        self.E = num_experts
        self.E_local = num_experts // self.world
        if w13.shape[0] != self.E_local or w2.shape[0] != self.E_local:
            raise ValueError(f"expected {self.E_local} local experts, got {w13.shape[0]}/{w2.shape[0]}")
        self.w13, self.w2, self.scales = w13, w2, scales
        self.ops = ops or CudaOps()

    def __call__(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        k = topk_ids.shape[1]
        sorted_slots, slot_pos, gs, n_valid_dev = self.ops.sort_slots(topk_ids, self.E)
        per_dest = gs.to(torch.int64).view(self.world, self.E_local)
        recv_expert = torch.empty_like(per_dest)
        dist.all_to_all_single(recv_expert, per_dest, group=self.group)
        # the send rows do not depend on what other ranks send: gather them
        # (up to the device-side valid count) while the counts travel
        x_send_all = self.ops.gather(x, sorted_slots, k, T * k, rows_dev=n_valid_dev)
        counts = torch.stack([per_dest.sum(1), recv_expert.sum(1)]).cpu()  # host split sizes (one sync)
        p = dict(send=counts[0].tolist(), recv=counts[1].tolist(), recv_expert=recv_expert, slot_pos=slot_pos)
        n_send, n_recv = sum(p["send"]), sum(p["recv"])
        x_send = x_send_all[:n_send]
        x_recv = x.new_empty((n_recv, H))
        dist.all_to_all_single(x_recv, x_send, p["recv"], p["send"], group=self.group)
        # received rows: grouped by source rank, then by local expert
        local_ids = torch.repeat_interleave(
            torch.arange(self.E_local, device=x.device, dtype=torch.int32).repeat(self.world),
            p["recv_expert"].reshape(-1).to(x.device)).to(torch.int32)
        if n_recv:
            o_recv = self.ops.expert_forward(x_recv, local_ids, self.w13, self.w2, self.scales)
        else:
            o_recv = x.new_empty((0, H))
        o_back = x.new_empty((n_send, H))
        dist.all_to_all_single(o_back, o_recv, p["send"], p["recv"], group=self.group)
        return self.ops.combine(o_back, p["slot_pos"], topk_weights.to(torch.float32).contiguous(), x.dtype)
