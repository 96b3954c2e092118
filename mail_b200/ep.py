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

Hot experts can be replicated (`replicas=`): every rank then also holds
their weights and serves the slots its own tokens route to them, so a
popular expert's load spreads over all ranks instead of landing on its
owner (ExpertPlacement).

The reference has no distributed code; this layer is what the multi-GPU
workloads need around the single-GPU hot path. The device work of steps 1, 3,
4 and 6 goes through `ops` (CudaOps = libmoe_b200 kernels); the collectives
are torch.distributed calls, so the exchange logic also runs with the gloo
backend on CPU tensors when `ops` is replaced (the CPU tests do that).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from . import moe as _moe


class ExpertPlacement:
    """Which rank runs each routed slot.

    E experts over W ranks: rank r owns experts [r * E / W, (r + 1) * E / W).
    `replicated` experts (the same list on every rank) are also held by every
    rank, and a slot routed to one of them runs on the rank whose token it
    is. The exchange then works in a virtual expert space of W * EL' ids,
    EL' = E / W + len(replicated): rank r's virtual experts
    [r * EL', (r + 1) * EL') are its owned experts in order, then its copies
    of the replicated ones in list order. `remap` turns this rank's global
    ids into virtual ids (invalid ids, < 0 or >= E, become -1: dropped), so
    the plan, dispatch and expert pass run unchanged over EL' local experts.
    Replicas hold the same weights, so each row's result is the same
    wherever it runs.
    """

    def __init__(self, num_experts: int, world: int, rank: int, replicated=()):
        if num_experts % world:
            raise ValueError("num_experts must be divisible by the world size")
        rep_list = [int(e) for e in replicated]
        if len(set(rep_list)) != len(rep_list) or any(e < 0 or e >= num_experts for e in rep_list):
            raise ValueError("replicated experts must be distinct ids in [0, num_experts)")
        self.E, self.world, self.rank = num_experts, world, rank
        self.replicated = rep_list
        self.EL = num_experts // world
        self.EL_virtual = self.EL + len(rep_list)
        self.E_virtual = world * self.EL_virtual
        lut = torch.empty(num_experts, dtype=torch.int32)
        for e in range(num_experts):
            owner = e // self.EL
            lut[e] = owner * self.EL_virtual + (e - owner * self.EL)
        for j, e in enumerate(rep_list):
            lut[e] = rank * self.EL_virtual + self.EL + j
        self._lut_cpu = lut
        self._lut = {}

    def lut(self, device) -> torch.Tensor:
        """Global id -> virtual id for this rank, on `device`."""
        key = str(device)
        if key not in self._lut:
            self._lut[key] = self._lut_cpu.to(device)
        return self._lut[key]

    def remap(self, topk_ids: torch.Tensor) -> torch.Tensor:
        if not self.replicated:
            return topk_ids
        ids = topk_ids.to(torch.int64)
        valid = (ids >= 0) & (ids < self.E)
        v = self.lut(topk_ids.device)[ids.clamp(0, self.E - 1)]
        return torch.where(valid, v, torch.full_like(v, -1)).to(torch.int32)

    def local_weights(self, w13, w2, scales=None, replicas=None):
        """This rank's owned experts followed by its replica copies, as one
        [EL', ...] set: logical (E, K, N) views over K-major storage (int8
        scales concatenated the same way)."""
        if not self.replicated:
            return w13, w2, scales
        if replicas is None:
            raise ValueError("replicated experts need their weights (replicas=)")
        ids, r13, r2 = replicas[0], replicas[1], replicas[2]
        rsc = replicas[3] if len(replicas) > 3 else None
        if [int(e) for e in ids] != self.replicated:
            raise ValueError("replica weights must be given in the order of the replicated ids")
        if r13.shape[0] != len(self.replicated) or r2.shape[0] != len(self.replicated):
            raise ValueError("one replica weight per replicated expert")
        w13v = torch.cat([_moe.kmajor(w13), _moe.kmajor(r13)]).transpose(1, 2)
        w2v = torch.cat([_moe.kmajor(w2), _moe.kmajor(r2)]).transpose(1, 2)
        sc = None
        if scales is not None:
            if rsc is None:
                raise ValueError("int8 replicas need their scales")
            sc = tuple(torch.cat([a.to(torch.float32), b.to(torch.float32)]) for a, b in zip(scales, rsc))
        return w13v, w2v, sc


def plan_replicas(counts: torch.Tensor, n: int):
    """Replicas that even out the expert-parallel load.

    counts [W, E]: slots rank r routes to expert e (the all-gathered
    per-rank counts, so every rank computes the same list). A rank's load is
    the slots of its owned experts from every rank plus its own slots to the
    replicated experts. Greedy: add, one at a time, the expert whose
    replication lowers the largest rank load the most (ties to the lower
    id); stop after n or when no single replica lowers it."""
    C = counts.to(torch.int64).cpu()
    W, E = C.shape
    EL = E // W
    tot = C.sum(0)
    owner = torch.arange(E) // EL
    load = torch.zeros(W, dtype=torch.int64).index_add_(0, owner, tot)
    chosen = []
    for _ in range(n):
        # max over ranks of the load if expert e were replicated, for every e
        cand = load.view(W, 1) + C - torch.nn.functional.one_hot(owner, W).T * tot.view(1, E)
        best = cand.max(0).values
        if chosen:
            best[torch.tensor(chosen)] = torch.iinfo(torch.int64).max
        e = int(torch.argmin(best))  # first minimum: the lower id on ties
        if int(best[e]) >= int(load.max()):
            break
        chosen.append(e)
        load = cand[:, e].clone()
    return chosen


def hot_experts(group_sizes: torch.Tensor, n: int):
    """The n experts with the most routed slots (ties to the lower id), from
    per-expert counts summed over the ranks — the replicas to place."""
    c = group_sizes.to(torch.int64).cpu()
    order = sorted(range(c.numel()), key=lambda e: (-int(c[e]), e))
    return order[:n]


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

    def combine(self, o_back, slot_pos, topk_weights, out_dtype, out=None):
        T, k = topk_weights.shape
        H = o_back.shape[1]
        y = out if out is not None else torch.empty((T, H), dtype=out_dtype, device=o_back.device)
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

    The batch is processed in `chunks` token chunks whose collectives are
    issued asynchronously on the communication stream: chunk c+1's dispatch
    overlaps chunk c's expert pass, and chunk c's return overlaps chunk c+1's
    expert pass. One host synchronisation per call (the split sizes).
    """

    def __init__(self, w13, w2, num_experts: int, scales=None, group=None, ops=None, chunks: int = 1,
                 min_chunk_tokens: int = 1024, replicas=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError("num_experts must be divisible by the world size")
        self.E = num_experts
        self.E_local = num_experts // self.world
        if w13.shape[0] != self.E_local or w2.shape[0] != self.E_local:
            raise ValueError(f"expected {self.E_local} local experts, got {w13.shape[0]}/{w2.shape[0]}")
        self.placement = ExpertPlacement(num_experts, self.world, self.rank, replicas[0] if replicas else ())
        self.w13, self.w2, self.scales = self.placement.local_weights(w13, w2, scales, replicas)
        self.ops = ops or CudaOps()
        self.chunks = max(1, int(chunks))
        self.min_chunk_tokens = min_chunk_tokens

    def _bounds(self, T: int):
        n = max(1, min(self.chunks, T // max(self.min_chunk_tokens, 1)))
        step = -(-T // n)
        return [(c, min(T, c + step)) for c in range(0, T, step)] or [(0, 0)]

    def __call__(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        k = topk_ids.shape[1]
        W, EL = self.world, self.placement.EL_virtual
        topk_weights = topk_weights.to(torch.float32).contiguous()
        topk_ids = self.placement.remap(topk_ids)  # virtual ids: replicated experts stay on this rank
        bounds = self._bounds(T)
        C = len(bounds)
        # 1. per-chunk dispatch plan (stable sort by expert = by owning rank)
        plans = [self.ops.sort_slots(topk_ids[a:b], self.placement.E_virtual) for a, b in bounds]
        per_dest = torch.stack([gs.to(torch.int64).view(W, EL) for _, _, gs, _ in plans], dim=1)  # [W, C, EL]
        recv_expert = torch.empty_like(per_dest)
        dist.all_to_all_single(recv_expert, per_dest.contiguous(), group=self.group)     # [W(src), C, EL]
        # 2. send rows: independent of what other ranks send, gathered while the counts travel
        x_send = [self.ops.gather(x[a:b], sl, k, (b - a) * k, rows_dev=nv)
                  for (a, b), (sl, _, _, nv) in zip(bounds, plans)]
        counts = torch.stack([per_dest.sum(2), recv_expert.sum(2)]).cpu()               # [2, W, C]: one sync
        send = [counts[0, :, c].tolist() for c in range(C)]
        recv = [counts[1, :, c].tolist() for c in range(C)]
        # 3. dispatch every chunk (asynchronous, in order on the communication stream)
        x_recv, d_work = [], []
        for c in range(C):
            buf = x.new_empty((sum(recv[c]), H))
            d_work.append(dist.all_to_all_single(buf, x_send[c][:sum(send[c])], recv[c], send[c],
                                                 group=self.group, async_op=True))
            x_recv.append(buf)
        # 4. local experts per chunk, each result sent back as soon as it exists
        ar = torch.arange(EL, device=x.device, dtype=torch.int32).repeat(W)
        o_back, r_work = [], []
        for c in range(C):
            d_work[c].wait()
            n_recv = x_recv[c].shape[0]
            if n_recv:
                local_ids = torch.repeat_interleave(ar, recv_expert[:, c, :].reshape(-1).to(x.device),
                                                    output_size=n_recv).to(torch.int32)
                o_recv = self.ops.expert_forward(x_recv[c], local_ids, self.w13, self.w2, self.scales)
            else:
                o_recv = x.new_empty((0, H))
            buf = x.new_empty((sum(send[c]), H))
            r_work.append(dist.all_to_all_single(buf, o_recv, send[c], recv[c], group=self.group, async_op=True))
            o_back.append(buf)
        # 5. weighted combine per chunk, straight into its rows of the output
        y = x.new_empty((T, H))
        for c, (a, b) in enumerate(bounds):
            r_work[c].wait()
            self.ops.combine(o_back[c], plans[c][1], topk_weights[a:b], x.dtype, out=y[a:b])
        return y


class PeerExpertParallelMoE:
    """Expert-parallel MoE MLP with the token exchange fused into the kernels.

    Each rank owns E / W experts. Token rows are stored by the dispatch
    kernel straight into the owning rank's receive buffer (CUDA IPC mapping,
    NVLink stores), and the down GEMM's epilogue stores each expert output
    row straight into the return buffer of the rank it came from; the
    collectives left are an all-gather of the [W, E] slot counts and two
    stream-ordered barriers. No host synchronisation per call.

    w13 / w2: this rank's experts (logical (E, K, N) layout, K-major storage,
    or int8 with scales=(w13_scale [E_local, 2I], w2_scale [E_local, H])).
    max_tokens: the largest T a call may pass (buffers are sized for every
    rank routing all its T * top_k slots to one rank).
    """

    def __init__(self, w13, w2, num_experts: int, max_tokens: int, top_k: int, dtype=torch.bfloat16,
                 scales=None, group=None, replicas=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError("num_experts must be divisible by the world size")
        self.E, self.EL = num_experts, num_experts // self.world
        if w13.shape[0] != self.EL or w2.shape[0] != self.EL:
            raise ValueError(f"expected {self.EL} local experts, got {w13.shape[0]}/{w2.shape[0]}")
        # from here on E / EL count virtual experts (owned + replicas per rank)
        self.placement = ExpertPlacement(num_experts, self.world, self.rank, replicas[0] if replicas else ())
        w13, w2, scales = self.placement.local_weights(w13, w2, scales, replicas)
        self.E, self.EL = self.placement.E_virtual, self.placement.EL_virtual
        self.H = w13.shape[1]
        self.I = w13.shape[2] // 2
        self.k = top_k
        self.max_tokens = max_tokens
        self.dtype = dtype
        self.quant = w13.dtype == torch.int8
        self.w13k, self.w2k = _moe.kmajor(w13), _moe.kmajor(w2)
        self.w_code = _moe._code(w13)
        self.s13 = self.s2 = None
        if self.quant:
            if scales is None:
                raise ValueError("int8 weights need scales")
            self.s13, self.s2 = (s.to(torch.float32).contiguous() for s in scales)
        self.device = w13.device
        self.x_code = _moe._DT[dtype]
        self.recv_code = _lib.I8 if self.quant else self.x_code
        S_max = max_tokens * top_k
        self.recv_cap = int(_lib.query("moe_align_capacity", self.world * S_max, self.EL, _moe.BLOCK_M))
        self.max_tiles = self.recv_cap // _moe.BLOCK_M
        esz = 1 if self.quant else torch.empty((), dtype=dtype).element_size()
        # IPC-shared buffers: receive rows, their scales (int8), row tags, return rows
        sizes = {"x": self.recv_cap * self.H * esz, "meta": self.recv_cap * 4, "ret": max(S_max, 1) * self.H * 2}
        if self.quant:
            sizes["scale"] = self.recv_cap * 4
        self._own, handles = {}, {}
        for name, nbytes in sizes.items():
            ptr, h = ctypes.c_void_p(), ctypes.create_string_buffer(64)
            _lib.call("moe_ipc_malloc", nbytes, ctypes.byref(ptr), h)
            self._own[name] = ptr.value
            handles[name] = h.raw
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        self._opened = []
        self.peer = {}
        for name in sizes:
            ptrs = []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(self._own[name])
                else:
                    p = ctypes.c_void_p()
                    _lib.call("moe_ipc_open", gathered[r][name], ctypes.byref(p))
                    self._opened.append(p.value)
                    ptrs.append(p.value)
            self.peer[name] = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.ret = _wrap(self._own["ret"], (max(S_max, 1), self.H), dtype, self.device)
        self.ws = _moe._workspace(_lib.query("moe_ep_expert_pass_workspace_size", self.recv_cap, self.I,
                                             self.recv_code), self.device)
        self.table = torch.empty(int(_lib.query("moe_tile_table_ints", self.EL, self.max_tiles)), dtype=torch.int32,
                                 device=self.device)
        self.dest_base = torch.empty(self.E, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.barrier(group=group)

    def _barrier(self):
        dist.all_reduce(self._flag, group=self.group)  # stream-ordered cross-rank barrier

    def __call__(self, x: torch.Tensor, topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
        T, H = x.shape
        if T > self.max_tokens or H != self.H or x.dtype != self.dtype or topk_ids.shape[1] != self.k:
            raise ValueError("PeerExpertParallelMoE: input does not match the buffers it was built for")
        st = _moe._stream(x.device)
        x = x.contiguous()
        ids = self.placement.remap(topk_ids.to(torch.int32)).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        S = T * self.k
        a = _moe.moe_align(ids, self.E, block_m=1)
        counts_all = torch.empty((self.world, self.E), dtype=torch.int32, device=x.device)
        dist.all_gather_into_tensor(counts_all, a["group_sizes"], group=self.group)
        ret_pos = torch.empty(max(S, 1), dtype=torch.int32, device=x.device)
        own_meta = self._own["meta"]
        _lib.call("moe_ep_plan", counts_all.data_ptr(), self.world, self.rank, self.E, a["slot_pos"].data_ptr(), S,
                  self.dest_base.data_ptr(), self.table.data_ptr(), self.max_tiles, own_meta, self.recv_cap,
                  ret_pos.data_ptr(), st)
        _lib.call("moe_ep_dispatch", x.data_ptr(), self.x_code, H, self.k, ids.data_ptr(),
                  a["sorted_slots"].data_ptr(), a["padded_offsets"].data_ptr(), self.dest_base.data_ptr(),
                  a["tile_table"][1:2].data_ptr(), S, self.world, self.rank, self.EL, self.recv_cap,
                  self.peer["x"].data_ptr(), self.recv_code,
                  self.peer["scale"].data_ptr() if self.quant else None, self.peer["meta"].data_ptr(),
                  self.err.data_ptr(), st)
        self._barrier()
        _lib.call("moe_ep_expert_pass", self._own["x"], self.recv_code, self._own.get("scale"), self.recv_cap, H,
                  self.w13k.data_ptr(), self.w2k.data_ptr(), self.EL, self.I, _moe._ptr(self.s13), _moe._ptr(self.s2),
                  self.table.data_ptr(), own_meta, self.peer["ret"].data_ptr(), self.world, self.ret.shape[0],
                  self.x_code, self.ws.data_ptr(), self.ws.numel(), st)
        self._barrier()
        y = torch.empty((T, H), dtype=x.dtype, device=x.device)
        if T:
            _lib.call("moe_combine_rows", self.ret.data_ptr(), self.x_code, H, ret_pos.data_ptr(), w.data_ptr(), T,
                      self.k, y.data_ptr(), self.x_code, st)
        return y

    def overflowed(self) -> bool:
        """True if a dispatch ever found its receive buffer too small (synchronises)."""
        return bool(self.err.item())

    def close(self):
        if not hasattr(self, "_own"):
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._opened:
            _lib.call("moe_ipc_close", p)
        self._opened = []
        dist.barrier(group=self.group)
        for p in self._own.values():
            _lib.call("moe_ipc_free", p)
        del self._own


def _wrap(ptr: int, shape, dtype, device) -> torch.Tensor:
    """A torch view of library-owned device memory (no ownership transfer)."""
    numel = 1
    for s in shape:
        numel *= s
    nbytes = numel * torch.empty((), dtype=dtype).element_size()
    return _from_ptr(ptr, nbytes, device).view(dtype).view(*shape)


def _from_ptr(ptr: int, nbytes: int, device) -> torch.Tensor:
    class _CudaArray:
        def __init__(self, p, n):
            self.__cuda_array_interface__ = {"shape": (n,), "typestr": "|u1", "data": (p, False), "version": 3}

    return torch.as_tensor(_CudaArray(ptr, nbytes), device=device)
