"""Expert-parallel sparse-MoE block exchanging over peer memory (NVLink).

The same partitioning as :class:`nki_moe_b200.ep.ExpertParallelMoE` (rank r
owns experts ``[r*E/P, (r+1)*E/P)``, each rank keeps its own tokens, one row
per (token, owning rank)), but the exchange is done by the library's own
kernels with stores into the other GPUs' memory instead of NCCL all-to-alls,
and the whole block is one stream-ordered library call per step with no host
synchronisation (``nkimoe_ep_peer_forward``):

    route -> sort (token, rank) pairs -> store rows into the owners' buffers
    -> wait for the P senders -> local experts over the received rows -> store
    each row's weighted sum back into its sender's buffer -> wait -> sum

Every rank allocates one exchange buffer with ``cudaMalloc`` and shares it by
CUDA IPC (handles swapped through the process group); no NVLink multicast
object is created.  Waits for peers are bounded on the device (~10 s) and
reported in the status word (``NKIMOE_SYNC_CHECK=1`` raises on it).

The reference leaves expert parallelism to NxDI (``moe_ep_degree``,
qwen.py:272, :515).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist
import torch.nn as nn

from . import ops
from ._lib import call, size_call

IPC_HANDLE_BYTES = 64


def plan_expert_replicas(load, world: int, extra_slots: int):
    """Copies of hot experts on lightly loaded ranks: a greedy plan that every
    rank computes identically from the same expected load.

    ``load``: expected rows per expert (length E, e.g. a routing histogram
    summed over the ranks, :func:`expert_load`).  Rank r owns experts
    ``[r*E/P, (r+1)*E/P)`` in its first E/P expert slots and has
    ``extra_slots`` more for copies.  A slot (t, k) of expert e goes to holder
    ``t mod n_e`` of its n_e holders, so rank r expects the sum over its slots
    of ``load[e] / n_e`` rows.  Each step puts a copy of the busiest rank's
    heaviest expert (per holder) on the least loaded rank with a free slot
    that does not hold it yet, as long as that lowers the sorted rank loads.

    Returns ``(slot_experts, holders)``: ``slot_experts[r]`` the expert of
    each of rank r's ``E/P + extra_slots`` slots (unused slots repeat the
    rank's first expert; nothing is routed to them) and ``holders[e]`` the
    slot ids ``rank * (E/P + extra_slots) + slot`` serving expert e, its
    owner's first."""
    load = [float(v) for v in load]
    E, P = len(load), int(world)
    if P < 1 or E % P or extra_slots < 0:
        raise ValueError("the experts must split evenly over the ranks; extra_slots >= 0")
    el = E // P
    per_rank = el + extra_slots
    slot_experts = [list(range(r * el, (r + 1) * el)) for r in range(P)]
    holders = [[(e // el, e % el)] for e in range(E)]

    def rank_loads(hs):
        rl = [0.0] * P
        for e in range(E):
            for r, _ in hs[e]:
                rl[r] += load[e] / len(hs[e])
        return rl

    scale = max(1.0, sum(load))

    def key(rl):  # sorted loads, busiest first, rounded against float noise
        return [round(v / scale, 12) for v in sorted(rl, reverse=True)]

    while True:
        rl = rank_loads(holders)
        free = [r for r in range(P) if len(slot_experts[r]) < per_rank]
        if not free:
            break
        busiest = max(range(P), key=lambda r: (rl[r], -r))
        cands = sorted((e for e in range(E) if any(r == busiest for r, _ in holders[e])),
                       key=lambda e: (-load[e] / len(holders[e]), e))
        placed = False
        for e in cands:
            held = {r for r, _ in holders[e]}
            targets = [r for r in free if r not in held]
            if not targets or load[e] <= 0:
                continue
            tgt = min(targets, key=lambda r: (rl[r], r))
            trial = [list(h) for h in holders]
            trial[e].append((tgt, len(slot_experts[tgt])))
            if key(rank_loads(trial)) < key(rl):
                holders = trial
                slot_experts[tgt].append(e)
                placed = True
                break
        if not placed:
            break
    for r in range(P):
        slot_experts[r] += [slot_experts[r][0]] * (per_rank - len(slot_experts[r]))
    return slot_experts, [[r * per_rank + j for r, j in h] for h in holders]


def expert_load(idx: torch.Tensor, num_experts: int, group=None) -> list:
    """Rows per expert in a routing ``idx [T, K]`` (this rank's tokens),
    summed over the process group when one is initialised: the same list on
    every rank, for :func:`plan_expert_replicas`."""
    counts = torch.bincount(idx.reshape(-1).long(), minlength=num_experts).to(torch.float64)
    if dist.is_available() and dist.is_initialized():
        g = group if group is not None else dist.group.WORLD
        if dist.get_world_size(g) > 1:
            counts = counts.to(idx.device)
            dist.all_reduce(counts, group=g)
    return counts.cpu().tolist()


class PeerExpertParallelMoE(nn.Module):
    """``forward(x [T, H]) -> [T, H]`` for this rank's ``T <= max_tokens``
    tokens.  Without an initialised process group (or with a group of one)
    it runs as a single rank that sends to itself."""

    def __init__(self, router_w: torch.Tensor, gate_up_local: torch.Tensor | None, down_local: torch.Tensor | None,
                 num_experts: int, top_k: int, max_tokens: int, group=None, router_bias: torch.Tensor | None = None,
                 device_epochs: bool = False, packed: ops.PackedExperts | None = None, replicas=None):
        """``gate_up_local [E/P, H, 2I]`` / ``down_local [E/P, I, H]``: this
        rank's experts in the reference layout; or ``packed``, the same experts
        already packed (``ops.PackedExperts``), with the two left ``None``.
        ``replicas``: a :func:`plan_expert_replicas` result, the same on every
        rank; the local weights are then the experts of this rank's slots
        (``slot_experts[rank]``, in that order)."""
        super().__init__()
        distributed = dist.is_available() and dist.is_initialized()
        self.group = (group if group is not None else dist.group.WORLD) if distributed else None
        self.world = dist.get_world_size(self.group) if distributed else 1
        self.rank = dist.get_rank(self.group) if distributed else 0
        local = packed.num_experts if packed is not None else gate_up_local.shape[0]
        if num_experts % self.world:
            raise ValueError("num_experts must split evenly over the ranks")
        if replicas is None:
            if local != num_experts // self.world:
                raise ValueError("local expert weights do not match num_experts / world size")
        else:
            slot_experts, holders = replicas
            if len(slot_experts) != self.world or len(holders) != num_experts or \
                    any(len(se) != local for se in slot_experts) or any(not h for h in holders):
                raise ValueError("replica plan does not match the ranks, experts or local weights")
        self.local_slots = local
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        self.num_experts, self.top_k, self.max_tokens = num_experts, top_k, max_tokens
        if packed is not None:
            self.device, self.hidden, self.inter = packed.w13.device, packed.hidden, packed.inter
        else:
            self.device = gate_up_local.device
            self.hidden = gate_up_local.shape[1]
            self.inter = gate_up_local.shape[2] // 2
        self.router_w = router_w.detach().float().contiguous()
        self.router_bias = router_bias.detach().float().contiguous() if router_bias is not None else None
        self.router_split = ops.router_split(self.router_w) if num_experts % 128 == 0 else None
        self.gate_up_local, self.down_local = gate_up_local, down_local
        self._packed = packed  # packed local weights given by the caller (the originals may be dropped)
        # device_epochs: every step's epoch is counted on the device (each
        # rank's buffer holds its count), so a captured step can be replayed
        self.device_epochs = device_epochs
        self.epoch = 0
        self._own = None
        self._opened = []
        self.replicas = replicas
        self.expert_slots = self.slot_counts = None
        self.max_holders = 0
        if replicas is not None:
            holders = replicas[1]
            self.max_holders = max(len(h) for h in holders)
            table = [h + [h[0]] * (self.max_holders - len(h)) for h in holders]
            self.expert_slots = torch.tensor(table, dtype=torch.int32, device=self.device)
            self.slot_counts = torch.tensor([len(h) for h in holders], dtype=torch.int32, device=self.device)
        self.bases = self._setup_buffers()

    @classmethod
    def from_dense(cls, moe, max_tokens: int, group=None, device_epochs: bool = False, extra_slots: int = 0,
                   expected_load=None):
        """Slice this rank's experts out of an ``NKIMoESimple`` holding all of
        them.  ``extra_slots > 0`` with ``expected_load`` (rows per expert,
        the same on every rank, e.g. :func:`expert_load` of a routing sample):
        each rank also holds copies of hot experts in up to ``extra_slots``
        more slots (:func:`plan_expert_replicas`)."""
        distributed = dist.is_available() and dist.is_initialized()
        g = (group if group is not None else dist.group.WORLD) if distributed else None
        world = dist.get_world_size(g) if distributed else 1
        rank = dist.get_rank(g) if distributed else 0
        el = moe.num_experts // world
        replicas = None
        if extra_slots > 0:
            if expected_load is None:
                raise ValueError("extra_slots needs expected_load")
            replicas = plan_expert_replicas(expected_load, world, extra_slots)
            sel = torch.tensor(replicas[0][rank], dtype=torch.long, device=moe.gate_up_proj.device)
        else:
            sel = torch.arange(rank * el, (rank + 1) * el, device=moe.gate_up_proj.device)
        return cls(moe.router.weight, moe.gate_up_proj.detach().index_select(0, sel).contiguous(),
                   moe.down_proj.detach().index_select(0, sel).contiguous(), moe.num_experts, moe.top_k, max_tokens,
                   group=g, router_bias=moe.router_bias, device_epochs=device_epochs, replicas=replicas)

    def packed(self):
        if self._packed is not None:
            return self._packed
        return ops.packed_experts(self.gate_up_local, self.down_local, "nxd")

    def _setup_buffers(self):
        nbytes = size_call("nkimoe_ep_peer_buffer_bytes", self.world, self.max_tokens, self.hidden, self.top_k)
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * IPC_HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            call("nkimoe_peer_alloc", nbytes, ctypes.byref(ptr), handle)
            self._own = ptr.value
            if self.world == 1:
                return [self._own]
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=self.group)
            bases = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    bases.append(self._own)
                    continue
                p = ctypes.c_void_p()
                hb = (ctypes.c_uint8 * IPC_HANDLE_BYTES).from_buffer_copy(h)
                call("nkimoe_peer_open", hb, ctypes.byref(p))
                self._opened.append(p.value)
                bases.append(p.value)
        return bases

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, return_routing: bool = False):
        """``out`` (optional): a contiguous bf16 ``[T, H]`` device tensor for
        the result.  With ``return_routing`` also returns this rank's routing
        ``(idx int32 [T, K], weights fp32 [T, K])``."""
        x = ops._contig(ops._cuda(x, "x"), torch.bfloat16)
        T, H = x.shape
        if T > self.max_tokens or H != self.hidden:
            raise ValueError(f"x [{T}, {H}] does not fit max_tokens {self.max_tokens} / hidden {self.hidden}")
        E, K, I, P = self.num_experts, self.top_k, self.inter, self.world
        pe = self.packed()
        if self.replicas is None:
            nbytes = size_call("nkimoe_ep_peer_workspace_bytes", T, H, I, E, K, P, self.max_tokens)
        else:
            nbytes = size_call("nkimoe_ep_peer_workspace_bytes_mapped", T, H, I, E, K, P, self.max_tokens,
                               self.local_slots)
        ws = ops.workspace(x.device, nbytes)
        if out is None:
            out = torch.empty(T, H, dtype=torch.bfloat16, device=x.device)
        elif out.dtype != torch.bfloat16 or tuple(out.shape) != (T, H) or not out.is_contiguous() or \
                out.device != x.device:
            raise ValueError("out must be a contiguous bf16 [T, H] tensor on x's device")
        idx = w = None
        if return_routing:
            idx = torch.empty(T, K, dtype=torch.int32, device=x.device)
            w = torch.empty(T, K, dtype=torch.float32, device=x.device)
        self.epoch = self.epoch % 0xFFFFFFFF + 1  # nonzero, increasing between steps
        epoch = 0 if self.device_epochs else self.epoch
        bases = (ctypes.c_void_p * P)(*self.bases)
        args = (ops._p(x), ops._p(self.router_w), ops._p(self.router_bias), ops._p(self.router_split), ops._p(pe.w13),
                ops._p(pe.w2), ops._p(out), ops._p(idx), ops._p(w), T, H, I, E, K, P, self.rank, self.max_tokens, bases,
                epoch, ops._p(ws), ws.numel(), ops._s(x))
        if self.replicas is None:
            call("nkimoe_ep_peer_forward", *args)
        else:
            call("nkimoe_ep_peer_forward_mapped", *args, self.local_slots, ops._p(self.expert_slots),
                 ops._p(self.slot_counts), self.max_holders)
        if ops.sync_check_enabled():
            ops.read_status(ws)
        return (out, idx, w) if return_routing else out

    def resync(self):
        """After a step that failed on some ranks (a rank that left a step, a
        wait that ran out), bring the ranks' step counters together again: every
        rank calls this between steps, with none of its exchange kernels in
        flight, and the next step runs with a fresh epoch on all of them.  Flags
        a failed step left in the buffers hold older epochs, so they are not
        taken for the next step's.  Host-counted epochs only."""
        if self.device_epochs:
            raise RuntimeError("resync needs host-counted epochs (device_epochs=False)")
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            t = torch.tensor([self.epoch], dtype=torch.int64, device=self.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            self.epoch = int(t.item())

    def forward_host(self, x: torch.Tensor, out: torch.Tensor | None = None,
                     done: torch.cuda.Event | None = None) -> torch.Tensor:
        """The block on a HOST batch ``x [T, H]`` (bf16, page-locked for the
        copies to overlap), the result returned into ``out`` (a new page-locked
        host tensor when None).  The copies run on two side streams of this
        module (one per direction) and use two device staging slots in turn,
        so a call's copy in overlaps the previous call's block and, with
        ``done``, its copy back overlaps the next call's block.

        ``done`` None: the current stream waits for the copy back.  ``done``
        an event: recorded when the copy back has completed; the current
        stream goes on without waiting, and ``out`` is ready after
        ``done.synchronize()`` (until then ``x`` and ``out`` must stay alive and
        untouched).  As with :meth:`forward`, every rank makes the call once per
        step.  The reference runs its block on host tensors in its module test
        (test_nki_moe.py:146-151)."""
        if x.is_cuda:
            raise ValueError("x must be a host tensor (forward takes device tensors)")
        x = ops._contig(x, torch.bfloat16)
        T, H = x.shape
        if T > self.max_tokens or H != self.hidden:
            raise ValueError(f"x [{T}, {H}] does not fit max_tokens {self.max_tokens} / hidden {self.hidden}")
        if out is None:
            out = torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True)
        elif out.is_cuda or out.dtype != torch.bfloat16 or tuple(out.shape) != (T, H) or not out.is_contiguous():
            raise ValueError("out must be a contiguous bf16 host tensor shaped like x")
        with torch.cuda.device(self.device):
            st = self._host_state()
            k = st["calls"] & 1
            st["calls"] += 1
            main = torch.cuda.current_stream(self.device)
            xd, yd = st["x"][k][:T], st["y"][k][:T]
            # copy in: after the block that last read this slot's rows
            st["in"].wait_event(st["x_free"][k])
            with torch.cuda.stream(st["in"]):
                xd.copy_(x, non_blocking=True)
                st["in_done"][k].record(st["in"])
            # block: after its rows arrived and this slot's last copy back
            main.wait_event(st["in_done"][k])
            main.wait_event(st["out_free"][k])
            self.forward(xd, out=yd)
            st["x_free"][k].record(main)
            # copy back, after the block
            st["out"].wait_event(st["x_free"][k])
            with torch.cuda.stream(st["out"]):
                out.copy_(yd, non_blocking=True)
                st["out_free"][k].record(st["out"])
            if done is not None:
                done.record(st["out"])
            else:
                main.wait_event(st["out_free"][k])
        return out

    def _host_state(self):
        st = getattr(self, "_host", None)
        if st is None:
            Tm, H = self.max_tokens, self.hidden
            st = {"calls": 0, "in": torch.cuda.Stream(self.device), "out": torch.cuda.Stream(self.device),
                  "x": [torch.empty(Tm, H, dtype=torch.bfloat16, device=self.device) for _ in range(2)],
                  "y": [torch.empty(Tm, H, dtype=torch.bfloat16, device=self.device) for _ in range(2)],
                  "x_free": [torch.cuda.Event() for _ in range(2)], "out_free": [torch.cuda.Event() for _ in range(2)],
                  "in_done": [torch.cuda.Event() for _ in range(2)]}
            self._host = st
        return st

    def close(self):
        """Unmap the peers' buffers and free this rank's (after every rank is
        done with the exchange)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                call("nkimoe_peer_close", ctypes.c_void_p(p))
            call("nkimoe_peer_free", ctypes.c_void_p(self._own))
        self._opened, self._own = [], None
