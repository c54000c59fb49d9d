"""Fully-sharded data-parallel training engine (ZeRO-3) for the block-diffusion step.

Units: the embedding table, each decoder layer, and the head (final norm, plus lm_head when it
is not tied to the embedding). A unit's parameters live flattened, in module order, in one bf16
buffer; rank r owns elements [r*S, (r+1)*S) (S = ceil(numel / world)) together with their fp32
master copy and fp32 AdamW moments.

Per step and per layer unit:
  forward   all-gather the unit into one of two gathered buffers (the next unit's gather is issued
            on the communication stream while this one computes), run the layer under no_grad,
            keep only its input (activation checkpointing);
  backward  re-gather (prefetching the previous layer), recompute the layer with grad enabled on
            leaf views of the gathered buffer whose .grad are pre-set views of one flat gradient
            buffer (autograd accumulates in place), then reduce-scatter the flat gradient.
Weight groups that one GEMM consumes (GDN qkv|z|b|a, attention q|k|v, MLP gate|up) are adjacent
in the flat buffer, so each is ONE leaf and one contiguous slice -- no concatenation copies.
After backward, one fused AdamW launch per unit updates the fp32 master shard and rewrites the
bf16 shard; the clip coefficient is computed on the device from one all-reduced scalar, so the
step has no host synchronisation.

Communication. On CUDA with more than one rank the engine keeps every parameter shard and both
flat gradient buffers in a symmetric peer heap (`parallel/peer.py`): a gather is one launch that
reads the peers' shards over NVLink into the gathered buffer, and a gradient reduce-scatter is one
launch that reads the peers' gradient slices, sums them in fp32, scales by 1/world, writes the
fp32 gradient shard and accumulates its sum of squares for the clip; it runs on the communication
stream, overlapped with the next layer's backward (the two gradient buffers alternate). The
global norm is one peer all-reduce launch; after the AdamW launches each rank publishes a
parameter epoch that the next step's gathers wait for. Set BDLLM_COMM=nccl (or run on CPU/gloo)
for the same steps over torch.distributed collectives.

This replaces the reference's FSDP2 wrapping of a `LayerStep` (`fsdp_train.py:86-171`): the
state fork calls submodules directly, which FSDP hooks cannot see (`fsdp_train.py:3-10`); here
parameters are gathered explicitly per unit, so there is no hook to bypass. Reduction semantics
match the reference: each rank's loss is its CE sum over the GLOBAL target count and gradients
are averaged over ranks (`fsdp_train.py:39-44,162,207-221`), so AdamW sees
(1/world) * grad(global mean CE), as in the reference.
"""

from __future__ import annotations

import os
import sys

import torch
import torch.distributed as dist

from .. import ops
from ..models.blockdiff import BreakMode, layer_step, rope_tables
from ..utils.trace import nvtx

# weight groups consumed by one GEMM: attribute set on the submodule -> member parameter names
FUSED_GROUPS = {
    "linear_attn": ("fused_in_weight", ("in_proj_qkv.weight", "in_proj_z.weight", "in_proj_b.weight",
                                        "in_proj_a.weight")),
    "self_attn": ("fused_qkv_weight", ("q_proj.weight", "k_proj.weight", "v_proj.weight")),
    "mlp": ("fused_gate_up_weight", ("gate_proj.weight", "up_proj.weight")),
}


SMALL_NUMEL = 1 << 20


def flat_order(module: torch.nn.Module) -> list:
    """Unique (name, parameter) of a unit in flat-buffer order: parameters below 1M elements that
    are not members of a fused weight group first (norm weights, conv taps, gate constants: what a
    layer reads outside its GEMMs), then the rest in module order. The small region is gathered
    before a layer runs; each GEMM weight after it can then be gathered by its own GEMM."""
    members = {m for _, (_, ms) in FUSED_GROUPS.items() for m in ms}
    uniq, seen = [], set()
    for n, p in module.named_parameters():
        if id(p) not in seen:
            seen.add(id(p))
            uniq.append((n, p))

    def is_member(n):
        return any(n == m or n.endswith("." + m) for m in members)

    small = [(n, p) for n, p in uniq if p.numel() < SMALL_NUMEL and not is_member(n)]
    ids = {id(p) for _, p in small}
    return small + [(n, p) for n, p in uniq if id(p) not in ids]


def _world():
    return (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)


def choose_saved_layers(per: list, per_act: list, free: float, frac: float = 0.92, reserve: int = 3 << 30):
    """How many leading layers keep their GEMM outputs: the budget is `frac` of `free` bytes less
    `reserve`. When every layer fits with its MLP activation too (`per_act` bytes each), keep it;
    otherwise count with `per` (gate|up only). Returns (layers, bytes used, keep_act)."""
    budget = frac * (free - reserve)
    keep_act = sum(per_act) < budget
    sizes = per_act if keep_act else per
    n, used = 0, 0
    while n < len(sizes) and used + sizes[n] < budget:
        used += sizes[n]
        n += 1
    return n, used, keep_act


class Unit:
    """A flat, sharded group of parameters of one module."""

    def __init__(self, name: str, module: torch.nn.Module, world: int, rank: int, device, dtype=torch.bfloat16,
                 alloc=None):
        self.name, self.world, self.rank, self.device = name, world, rank, device
        self.entries = []  # (param name, shape, offset, numel), flat_order
        off = 0
        for pname, p in flat_order(module):
            self.entries.append((pname, tuple(p.shape), off, p.numel()))
            off += p.numel()
        self.small_numel = sum(k for n, _, _, k in self.entries if self._is_small(n, k))  # a prefix
        self.numel = off
        self.shard = (off + world - 1) // world
        if world > 1:  # 16-byte aligned slices of bf16 and fp32 buffers for the peer kernels
            self.shard = (self.shard + 63) // 64 * 64
        self.padded = self.shard * world
        if alloc is not None:  # in the symmetric heap: peers read it directly
            self.p, self.p_off = alloc(self.shard, dtype)
        else:
            self.p, self.p_off = torch.zeros(self.shard, dtype=dtype, device=device), None
        self.master = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.m = torch.zeros(self.shard, dtype=torch.float32, device=device)
        self.v = torch.zeros(self.shard, dtype=torch.float32, device=device)
        # the reduce-scattered gradient: fp32 when ranks are summed, the local (model dtype)
        # gradient itself at world 1 (no reduction, and half the memory of an fp32 copy)
        self.g = torch.zeros(self.shard, dtype=torch.float32 if world > 1 else dtype, device=device)
        self.groups = self._groups()

    @staticmethod
    def _is_small(name: str, numel: int) -> bool:
        members = {m for _, (_, ms) in FUSED_GROUPS.items() for m in ms}
        return numel < SMALL_NUMEL and not any(name == m or name.endswith("." + m) for m in members)

    def _groups(self):
        """Fused groups present in this unit: (submodule path, attr, first offset, numel, rows, cols)."""
        by_name = {n: (s, o, k) for n, s, o, k in self.entries}
        out = []
        for n, _, _, _ in self.entries:
            for kind, (attr, members) in FUSED_GROUPS.items():
                pre = n.split(kind + ".")[0] + kind + "." if (kind + ".") in n else None
                if pre is None or n != pre + members[0]:
                    continue
                names = [pre + m for m in members]
                if not all(x in by_name for x in names):
                    continue
                offs = [by_name[x][1] for x in names]
                sizes = [by_name[x][2] for x in names]
                if any(offs[i] + sizes[i] != offs[i + 1] for i in range(len(offs) - 1)):
                    continue
                cols = by_name[names[0]][0][1]
                rows = sum(by_name[x][0][0] for x in names)
                out.append((pre[:-1], attr, offs[0], sum(sizes), rows, cols))
        return out

    @torch.no_grad()
    def load_full(self, flat: torch.Tensor) -> None:
        lo = self.rank * self.shard
        hi = min(self.numel, lo + self.shard)
        self.master.zero_()
        if hi > lo:
            self.master[: hi - lo].copy_(flat[lo:hi].to(self.device, torch.float32))
        self.p.copy_(self.master)

    def flat_of(self, module: torch.nn.Module) -> torch.Tensor:
        own = dict(module.named_parameters())
        return torch.cat([own[n].detach().reshape(-1) for n, _, _, _ in self.entries])

    def views(self, buf: torch.Tensor) -> dict:
        return {n: buf[o : o + k].view(s) for n, s, o, k in self.entries}

    def gather_into(self, out: torch.Tensor) -> None:
        if self.world == 1:
            out[: self.shard].copy_(self.p)
        else:
            dist.all_gather_into_tensor(out[: self.padded], self.p)

    def reduce_scatter_from(self, flat_grad: torch.Tensor) -> None:
        """flat_grad [>= padded] -> self.g (fp32), averaged over ranks (overwrites self.g)."""
        src = flat_grad[: self.padded]
        if self.world == 1:
            self.g.copy_(src[: self.shard])
        else:
            dist.reduce_scatter_tensor(self.g, src.float() if src.dtype != torch.float32 else src,
                                       op=dist.ReduceOp.AVG)


class FSDPEngine:
    """Sharded training of a `BlockDiffusionLM`.

    `model` must hold the initial weights (identical on every rank, e.g. `build_model` with one
    seed); the engine copies each rank's shards and then releases the model's parameter storage
    (the module tree stays, on the meta device, as the structure the layer code reads)."""

    def __init__(self, model, *, lr: float = 1e-5, betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0,
                 grad_clip: float = 1.0):
        self.cfg = model.config
        self.world, self.rank = _world()
        p0 = next(model.parameters())
        self.device, self.dtype = p0.device, p0.dtype
        self.lr, self.betas, self.eps, self.wd, self.grad_clip = lr, betas, eps, weight_decay, grad_clip
        self.step_count = 0
        tm = model.text_model
        self.tied = self.cfg.tie_word_embeddings
        head_mod = torch.nn.ModuleDict({"norm": tm.norm} if self.tied else {"norm": tm.norm, "lm_head": model.lm_head})
        mods = [("embed", tm.embed_tokens)] + [(f"layers.{i}", tm.layers[i]) for i in range(self.cfg.num_hidden_layers)]
        mods.append(("head", head_mod))
        self.peer = None
        if self.world > 1 and self.device.type == "cuda" and os.environ.get("BDLLM_COMM", "peer") == "peer":
            from .peer import SymmetricHeap

            self.peer = SymmetricHeap(self._heap_bytes([m for _, m in mods]), self.device)
        alloc = self.peer.alloc if self.peer is not None else None
        mk = lambda name, mod: Unit(name, mod, self.world, self.rank, self.device, self.dtype, alloc)  # noqa: E731
        self.units = [mk(name, mod) for name, mod in mods]
        self.embed, self.layers, self.head = self.units[0], self.units[1:-1], self.units[-1]
        for u, (_, mod) in zip(self.units, mods):
            u.load_full(u.flat_of(mod))
        self.model = model.to("meta")
        if self.tied:
            self.model.lm_head.weight = self.model.text_model.embed_tokens.weight
        n = max(u.padded for u in self.units) if self.world > 1 else 0
        self.bufs = [torch.empty(n, dtype=self.dtype, device=self.device) for _ in range(2)]
        self.owner = [None, None]
        self.ready = [None, None]
        self.lru = 0
        gmax = max(u.padded for u in self.layers + [self.head])
        if self.peer is not None:  # two alternating gradient buffers: one is reduce-scattered while
            # the next layer's backward fills the other
            self.grads, self.grad_offs = zip(*[self.peer.alloc(gmax, self.dtype) for _ in range(2)])
            # untied: the table gradient in the model dtype, written as sorted per-id sums (fp32 within
            # a rank, fp32 across ranks in the reduce-scatter), like every other unit's gradient
            self.table_grad, self.table_off = self.peer.alloc(self.embed.padded,
                                                              torch.float32 if self.tied else self.dtype)
        elif self.world == 1:  # each unit's backward writes its own gradient (unit.g) in place
            self.grads = ()
            # untied: the embedding gradient is written per token id straight into embed.g (sorted
            # ids, fp32 sums per id), so no fp32 [V, D] table is needed (5 GB at the 27B shape)
            self.table_grad = torch.zeros(self.embed.padded, dtype=torch.float32, device=self.device) \
                if self.tied else None
        else:
            self.grads = (torch.empty(gmax, dtype=self.dtype, device=self.device),)
            self.table_grad = torch.zeros(self.embed.padded, dtype=torch.float32, device=self.device)
        # sum of squares of this rank's reduced gradient shards (the clip norm), filled as each unit's
        # gradient is reduced; summed over ranks once per step
        self.sq = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.sq_all = torch.zeros(1, dtype=torch.float32, device=self.device)
        self.grad_i = 0
        self.rs_done = [None] * len(self.grads)
        self.epoch = 0
        # fused all-gather -> first GEMM of each layer (peer heap only)
        self.fused_ag = self.peer is not None and os.environ.get("BDLLM_FUSED_AG", "1") != "0"
        if self.fused_ag:
            self.ag_ready = [torch.zeros(8192 + 64, dtype=torch.int32, device=self.device) for _ in range(2)]
            self.ag_claim = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.ag_seq = 0
            self._pending = None
        self.comm = torch.cuda.Stream(device=self.device) if self.device.type == "cuda" else None
        self.anchor = torch.zeros((), device=self.device, requires_grad=True)
        # keep the GDN core / attention outputs of the checkpointed forward for the backward's
        # recomputation (about 0.5 GB per GDN layer at L 4096: the fp32 block states)
        self.save_cores = self.device.type == "cuda" and os.environ.get("BDLLM_SAVE_CORES", "1") != "0"
        if self.save_cores:
            from ..ops import cuda as Cu

            self.act_store = Cu.ActStore
        # also keep the GEMM outputs of the checkpointed forward: "1" every layer, "0" none, "<n>" the
        # first n layers, or "auto": as many layers as fit in free memory, decided at the first step
        # from the row count
        self.save_gemms = os.environ.get("BDLLM_SAVE_GEMMS", "auto") if self.save_cores else "0"
        self.keep_act = False  # whether the kept MLP outputs include the activation (decided with them)
        # which pass is gathering: in the backward, a layer whose GEMM outputs were kept reruns none
        # of its GEMMs, so its gather cannot ride on one and takes the prefetched peer gather instead
        self.phase = "fwd"
        self.layer_index = {id(u): j for j, u in enumerate(self.layers)}
        if self.peer is not None:  # every shard written before any peer reads one
            torch.cuda.synchronize(self.device)
            dist.barrier()

    def _heap_bytes(self, modules) -> int:
        """Bytes of the symmetric heap: every unit's bf16 shard, two bf16 gradient buffers of the
        largest layer/head unit and the embedding-table gradient (fp32 when the head is tied to the
        table, else the model dtype), each 256-byte aligned."""
        w = self.world
        esz = torch.empty(0, dtype=self.dtype).element_size()

        def shard(mod):
            n = sum(p.numel() for p in {id(p): p for p in mod.parameters()}.values())
            return ((n + w - 1) // w + 63) // 64 * 64

        a = lambda b: (b + 255) // 256 * 256  # noqa: E731
        shards = [shard(m) for m in modules]
        total = sum(a(s * esz) for s in shards)
        total += 2 * a(max(shards[1:]) * w * esz)
        total += a(shards[0] * w * (4 if self.tied else esz))  # the embedding-table gradient
        return total + 4096

    # ------------------------------------------------------------------ gathers
    def _fused_plan(self, unit: Unit):
        """Byte size of the unit's small-parameter prefix when its GEMM weights can be gathered by
        their own GEMMs (layer units), else None."""
        plan = getattr(unit, "_ag_plan", False)
        if plan is False:
            plan = None
            if any(g[1] in ("fused_in_weight", "fused_qkv_weight") for g in unit.groups):
                plan = unit.small_numel * unit.p.element_size()
            unit._ag_plan = plan
        return plan

    def _fused_for(self, unit: Unit) -> bool:
        """Gather `unit` inside its first GEMM? Every layer in the forward (it runs all its GEMMs);
        in the backward only layers whose GEMM outputs were not kept (their recomputation reruns
        the projection GEMMs)."""
        if not self.fused_ag or self._fused_plan(unit) is None:
            return False
        j = self.layer_index.get(id(unit))
        return not (self.phase == "bwd" and j is not None and self.gemm_saved(j))

    def gather(self, unit: Unit, prefetch: bool = False) -> torch.Tensor:
        if self.world == 1:  # the shard is the whole unit
            return unit.p
        if self._fused_for(unit):
            return self._gather_fused(unit, prefetch)
        for i in range(2):
            if self.owner[i] is unit:
                if self.ready[i] is not None:
                    torch.cuda.current_stream(self.device).wait_event(self.ready[i])
                    self.ready[i] = None
                self.lru = 1 - i
                return self.bufs[i]
        i = self.lru
        self.lru = 1 - i
        self.owner[i] = unit
        buf = self.bufs[i]
        if prefetch and self.comm is not None:
            self.comm.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.comm):
                self.gather_into(unit, buf)
                ev = torch.cuda.Event()
                ev.record(self.comm)
            self.ready[i] = ev
        else:
            self.gather_into(unit, buf)
            self.ready[i] = None
        return buf

    def _gather_fused(self, unit: Unit, prefetch: bool) -> torch.Tensor:
        """Fused path: the small-parameter prefix (norm weights, conv taps, gate constants) is
        copied now; every GEMM weight of the unit is gathered by the first GEMM that reads it
        (`_C.gemm_ag`), tile by tile, while that GEMM computes."""
        if prefetch:
            return None  # nothing to prefetch: the gathers happen inside the GEMMs
        for i in range(2):
            if self.owner[i] is unit and self._pending is None:
                self.lru = 1 - i
                return self.bufs[i]
        self.check_gathered()
        i = self.lru
        self.lru = 1 - i
        self.owner[i] = unit
        buf = self.bufs[i]
        esz = buf.element_size()
        sb = unit.shard * esz
        small = self._fused_plan(unit)
        if small:
            self.peer.gather_range(unit.p_off, sb, buf, 0, small, self.epoch)
        # the GEMM weights still to gather: (byte lo, byte hi)
        todo = []
        for n, _, o, k in unit.entries:
            if o * esz >= small:
                todo.append((o * esz, (o + k) * esz))
        for path, attr, off, numel, rows, cols in unit.groups:  # a fused group is one weight
            todo = [r for r in todo if not (off * esz <= r[0] < (off + numel) * esz)]
            todo.append((off * esz, (off + numel) * esz))
        pending = {lo: hi for lo, hi in todo}
        base = buf.data_ptr()
        ready = self.ag_ready[i]
        C, peer = self.peer.C, self.peer

        def hook(a, w, out, epi, gu):
            lo = w.data_ptr() - base
            hi = pending.get(lo)
            if hi is None or hi != lo + w.numel() * esz:
                return False
            self.ag_seq += 1
            C.gemm_ag(a, w, out, epi, gu, peer.ptrs, peer.rank, unit.p_off, sb, buf, ready, self.ag_claim,
                      self.ag_seq, self.epoch, 0, peer.timeout, lo, hi)
            del pending[lo]
            if not pending:
                from ..ops import cuda as Cu

                Cu.AG_HOOK[0] = None
                self._pending = None
            return True

        from ..ops import cuda as Cu

        self._pending = (unit, pending)
        Cu.AG_HOOK[0] = hook
        return buf

    def check_gathered(self) -> None:
        """Raise if a layer ran without gathering all of its GEMM weights (the buffer would be
        incomplete for the next use)."""
        if self.fused_ag and self._pending is not None:
            from ..ops import cuda as Cu

            Cu.AG_HOOK[0] = None
            (unit, left), self._pending = self._pending, None
            raise RuntimeError(f"fused all-gather of {unit.name}: {len(left)} weights were never read by a GEMM")

    def gather_into(self, unit: Unit, out: torch.Tensor) -> None:
        if self.peer is not None:
            self.peer.all_gather(unit.p_off, unit.shard * unit.p.element_size(), out, self.epoch)
        else:
            unit.gather_into(out)

    def grad_buffer(self, unit: Unit) -> torch.Tensor:
        """A zeroed flat gradient buffer for `unit` (waits until its previous reduce-scatter ended).
        One rank: the unit's own gradient tensor, which the optimizer reads directly."""
        if not self.grads:
            unit.g.zero_()
            return unit.g
        j = self.grad_i
        self.grad_i = (j + 1) % len(self.grads)
        if self.rs_done[j] is not None:
            torch.cuda.current_stream(self.device).wait_event(self.rs_done[j])
            self.rs_done[j] = None
        g = self.grads[j][: unit.padded]
        g.zero_()
        return g

    def reduce_scatter(self, unit: Unit, flat_grad: torch.Tensor) -> None:
        if self.peer is None:
            if flat_grad.data_ptr() == unit.g.data_ptr():  # one rank: the gradient is already in place
                ops.sumsq_(flat_grad[: unit.shard], self.sq)
            elif self.world == 1:  # the model-dtype copy and its sum of squares in one pass
                ops.sumsq_(flat_grad[: unit.shard], self.sq, unit.g)
            else:
                unit.reduce_scatter_from(flat_grad)
                ops.sumsq_(unit.g, self.sq)
            return
        if self.table_grad is not None and flat_grad.data_ptr() == self.table_grad.data_ptr():
            j, off, f32 = None, self.table_off, self.table_grad.dtype == torch.float32
        else:
            j = next(k for k, g in enumerate(self.grads) if g.data_ptr() == flat_grad.data_ptr())
            off, f32 = self.grad_offs[j], False
        self.comm.wait_stream(torch.cuda.current_stream(self.device))
        adam = None
        if not self.grad_clip:  # no global clip: AdamW runs inside the reduce-scatter, overlapped
            b1, b2 = self.betas
            adam = ((unit.master, unit.m, unit.v, unit.p),
                    (self.lr, b1, b2, self.eps, self.wd, 1 - b1 ** self.step_count, 1 - b2 ** self.step_count))
        with torch.cuda.stream(self.comm), nvtx(f"rs.{unit.name}"):
            self.peer.reduce_scatter(off, unit.shard, f32, unit.g, 1.0 / self.world, self.sq, adam=adam)
            if j is not None:
                ev = torch.cuda.Event()
                ev.record(self.comm)
                self.rs_done[j] = ev

    # ------------------------------------------------------------------ layer parameter binding
    def leaves(self, unit: Unit, buf: torch.Tensor, grad: torch.Tensor | None):
        """Parameter tensors for `unit` over gathered `buf`. With `grad`, fused groups and the other
        parameters are leaves whose .grad are views of `grad` (autograd accumulates in place).
        Returns (params by name, fused attrs {submodule path: (attr, tensor)})."""
        params, fused = {}, {}
        for path, attr, off, numel, rows, cols in unit.groups:
            t = buf[off : off + numel].view(rows, cols)
            if grad is not None:
                t = t.detach().requires_grad_(True)
                t.grad = grad[off : off + numel].view(rows, cols)
            fused[path] = (attr, t)
            for n, s, o, k in unit.entries:
                if off <= o < off + numel:
                    params[n] = t.detach()[(o - off) // cols : (o - off + k) // cols].view(s) if grad is not None \
                        else buf[o : o + k].view(s)
        for n, s, o, k in unit.entries:
            if n in params:
                continue
            t = buf[o : o + k].view(s)
            if grad is not None:
                t = t.detach().requires_grad_(True)
                t.grad = grad[o : o + k].view(s)
            params[n] = t
        return params, fused

    # ------------------------------------------------------------------ step
    def forward_hidden(self, x0_2, xt_2, block: int, fault: BreakMode | None = None):
        fault = fault or BreakMode()
        B, L = x0_2.shape
        ids = torch.cat([xt_2, x0_2], 1)
        h = _EmbedFn.apply(ids, self.anchor, self)
        cos, sin = rope_tables(self.cfg, L, self.dtype, ids.device)
        for i in range(len(self.layers)):
            h = _LayerFn.apply(h, self.anchor, self, i, L, block, cos, sin, fault)
        return h

    def step(self, x0, prompt_len, valid_len, *, block: int, mask_id: int, n_local: int, n_global, gstep: int):
        """One optimizer step on this rank's rows (already on the device). n_local: this rank's
        scored-target count (host int); n_global: the global count (python number or 0-d device
        tensor). Returns this rank's loss contribution (device tensor); summed over ranks it is the
        global mean CE.

        On one rank, when the number of layers keeping GEMM outputs was chosen from the probe step
        and the step then runs out of memory before its update, the step is run again with two
        layers fewer (the masks come from the step's seed, so it is the same step)."""
        kw = dict(block=block, mask_id=mask_id, n_local=n_local, n_global=n_global, gstep=gstep)
        try:
            return self._step(x0, prompt_len, valid_len, **kw)
        except torch.cuda.OutOfMemoryError:
            if self.world > 1 or not self.save_gemms.isdigit() or not getattr(self, "_auto_saved", False) \
                    or self._updated:
                raise
            n = len(self.layers) if self.save_gemms == "1" else int(self.save_gemms)
            if n == 0:
                raise
            self.save_gemms = str(max(0, n - 2))
            self.act_store.clear()
            self.step_count -= 1
            torch.cuda.empty_cache()
            print(f"[fsdp] out of memory with GEMM outputs kept for {n} layers; retrying with "
                  f"{self.save_gemms}", file=sys.stderr, flush=True)
            return self._step(x0, prompt_len, valid_len, **kw)

    def _step(self, x0, prompt_len, valid_len, *, block: int, mask_id: int, n_local: int, n_global, gstep: int):
        from ..train.objective import complementary_step_inputs

        self._updated = False
        self.step_count += 1
        gen = torch.Generator(device=self.device).manual_seed(gstep * 1000 + self.rank)
        x0_2, xt_2, m_2 = complementary_step_inputs(x0, prompt_len, block, mask_id, gen, valid_len,
                                                    seed=gstep * 1000 + self.rank)
        probe = self.save_gemms == "auto"  # this step keeps no GEMM outputs and measures the peak
        if probe:
            torch.cuda.synchronize(self.device)
            torch.cuda.reset_peak_memory_stats(self.device)
        self.phase = "fwd"
        h = self.forward_hidden(x0_2, xt_2, block)
        L = x0.shape[1]
        if self.table_grad is not None and self.table_grad.dtype == torch.float32:  # (others: zeroed in backward)
            self.table_grad.zero_()
        self.sq.zero_()
        loss = _HeadFn.apply(h[:, :L], m_2, x0_2, self.anchor, self, n_global, n_local)
        loss.backward()
        self._updated = True  # from here on the step has changed the weights: no retry
        self._optimizer_step()
        if probe:
            self._decide_save_gemms(x0_2.shape[0] * 2 * x0_2.shape[1])
            self._auto_saved = True
        return loss.detach()

    def gemm_bytes_per_layer(self, rows: int, with_act: bool = False) -> list:
        """Bytes the saved GEMM outputs of each layer take for one step of `rows` token rows (the MLP
        activation included only with `with_act`; without it the backward rebuilds it)."""
        c = self.cfg
        mlp = c.hidden_size + (3 if with_act else 2) * c.intermediate_size  # down output, gate|up[, act]
        out = []
        for t in c.layer_types[: len(self.layers)]:
            if t == "linear_attention":
                proj = c.conv_dim + c.value_dim + 2 * c.linear_num_value_heads
            else:
                proj = 2 * c.num_attention_heads * c.head_dim + 2 * c.num_key_value_heads * c.head_dim
            out.append(rows * (proj + c.hidden_size + mlp) * 2)
        return out

    def gemm_bytes_per_step(self, rows: int) -> int:
        """Bytes the saved GEMM outputs of every layer take for one step of `rows` token rows."""
        return sum(self.gemm_bytes_per_layer(rows))

    def gemm_saved(self, i: int) -> bool:
        """Whether layer i keeps its GEMM outputs across checkpointing."""
        s = self.save_gemms
        return s == "1" or (s.isdigit() and s != "0" and i < int(s))

    def _decide_save_gemms(self, rows: int) -> None:
        """After a step that kept no GEMM outputs: keep those of as many layers (from the first,
        whose outputs live longest) as fit in 92 % of the device memory that the step's peak left
        unreserved, less 3 GiB. The caching allocator keeps its peak reservation, so what the saved
        outputs add has to come from memory that is still free now. Every rank takes the same
        decision: the smallest headroom over ranks counts. With several ranks a step that runs out
        of memory cannot be rerun (the other ranks are inside their collectives), so the budget
        there is the wider-margin 85 % less 2 GiB."""
        per = self.gemm_bytes_per_layer(rows)
        torch.cuda.synchronize(self.device)
        free = torch.tensor([float(torch.cuda.mem_get_info(self.device)[0])], device=self.device)
        if self.world > 1:
            dist.all_reduce(free, op=dist.ReduceOp.MIN)
        margin = dict(frac=0.85, reserve=2 << 30) if self.world > 1 else {}
        n, used, self.keep_act = choose_saved_layers(per, self.gemm_bytes_per_layer(rows, with_act=True),
                                                     float(free[0]), **margin)
        if self.keep_act:
            per = self.gemm_bytes_per_layer(rows, with_act=True)
        self.save_gemms = "1" if n == len(per) else str(n)
        if self.rank == 0:
            print(f"[fsdp] GEMM outputs across checkpointing: kept for {n} of {len(per)} layers "
                  f"({used / 2**30:.1f} of {sum(per) / 2**30:.1f} GiB; free {float(free[0]) / 2**30:.1f} GiB; "
                  f"MLP activation {'kept' if self.keep_act else 'rebuilt from gate|up'})",
                  file=sys.stderr, flush=True)

    @torch.no_grad()
    def _optimizer_step(self):
        if self.peer is not None:
            torch.cuda.current_stream(self.device).wait_stream(self.comm)
            self.peer.allreduce_f32(self.sq, self.sq_all)
            norm = self.sq_all[0].sqrt()
            if not self.grad_clip:  # the updates already ran inside the reduce-scatters
                self.last_grad_norm = norm
                self.invalidate()
                return
        else:
            if self.world > 1:
                dist.all_reduce(self.sq)
            norm = self.sq.sqrt()
        coef = torch.clamp(self.grad_clip / (norm + 1e-6), max=1.0) if self.grad_clip > 0 else torch.ones_like(norm)
        b1, b2 = self.betas
        bc1, bc2 = 1 - b1 ** self.step_count, 1 - b2 ** self.step_count
        for u in self.units:
            ops.adamw_flat(u.master, u.p, u.g, u.m, u.v, self.lr, b1, b2, self.eps, self.wd, coef, bc1, bc2)
        self.last_grad_norm = norm
        self.invalidate()

    def invalidate(self) -> None:
        """Forget gathered copies (their shards changed) and, with the peer heap, publish the new
        parameter epoch that peers' next gathers wait for."""
        if self.fused_ag:
            self.check_gathered()
        self.owner = [None, None]
        self.ready = [None, None]
        self.epoch += 1
        if self.peer is not None:
            self.peer.publish_epoch(self.epoch)

    def close(self) -> None:
        """Release the peer heap (collective; the engine is unusable afterwards)."""
        if self.peer is not None:
            torch.cuda.synchronize(self.device)
            dist.barrier()
            self.peer.close()
            self.peer = None

    # ------------------------------------------------------------------ inspection
    @torch.no_grad()
    def full_state(self) -> dict:
        """Gather every unit's full bf16 parameters (collective). {our key: tensor} on this device."""
        out = {}
        prefixes = {"embed": "text_model.embed_tokens.", "head": ""}
        for u in self.units:
            buf = torch.empty(u.padded, dtype=self.dtype, device=self.device)
            self.gather_into(u, buf)
            for n, s, o, k in u.entries:
                if u.name == "head":
                    key = ("text_model." + n) if n.startswith("norm.") else n
                elif u.name == "embed":
                    key = prefixes["embed"] + n
                else:
                    key = f"text_model.{u.name}.{n}"
                out[key] = buf[o : o + k].view(s).clone()
        return out


# ---------------------------------------------------------------------------- autograd units


def _count_launch() -> None:
    """One launch of this repository's kernels, for the step's launch count."""
    from ..ops import cuda as Cu

    Cu.LAUNCHES[0] += 1


class _EmbedFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, anchor, engine):
        buf = engine.gather(engine.embed)
        table = engine.embed.views(buf)["weight"]
        if ids.is_cuda:
            from ..ops import _native

            h = _native.require().embed_fwd(ids.contiguous(), table)
            _count_launch()
        else:
            h = torch.nn.functional.embedding(ids, table)
        ctx.save_for_backward(ids)
        ctx.engine = engine
        if engine.layers:
            engine.gather(engine.layers[0], prefetch=True)
        return h

    @staticmethod
    def backward(ctx, dh):
        (ids,) = ctx.saved_tensors
        engine = ctx.engine
        V, D = engine.cfg.vocab_size, engine.cfg.hidden_size
        if engine.table_grad is None or engine.table_grad.dtype != torch.float32:
            # untied: per-id sums straight into the model-dtype gradient (one rank: embed.g; several
            # ranks on peer memory: the table that the reduce-scatter reads)
            g = engine.embed.g if engine.table_grad is None else engine.table_grad
            g.zero_()
            gt = g[: V * D].view(V, D)
            flat_ids = ids.reshape(-1)
            if gt.is_cuda:
                from ..ops import _native

                sid, perm = torch.sort(flat_ids, stable=True)  # fixed summation order within a run
                _native.require().embed_bwd_sorted(gt, sid, perm, dh.reshape(-1, D))
                _count_launch()
            else:
                acc = torch.zeros(V, D, dtype=torch.float32)
                acc.index_add_(0, flat_ids, dh.reshape(-1, D).float())
                gt.copy_(acc)
            engine.reduce_scatter(engine.embed, g)
            return None, None, None
        tg = engine.table_grad[: V * D].view(V, D)  # already holds the tied head's gradient, if any
        if tg.is_cuda:
            from ..ops import _native

            _native.require().embed_bwd_(tg, ids.reshape(-1).contiguous(), dh.reshape(-1, D))
            _count_launch()
        else:
            tg.index_add_(0, ids.reshape(-1), dh.reshape(-1, D).float())
        engine.reduce_scatter(engine.embed, engine.table_grad)
        return None, None, None


def _bind(layer, fused):
    for path, (attr, t) in fused.items():
        sub = layer.get_submodule(path) if path else layer
        object.__setattr__(sub, attr, t)


def _unbind(layer, fused):
    for path, (attr, _) in fused.items():
        sub = layer.get_submodule(path) if path else layer
        object.__delattr__(sub, attr)


class _LayerFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, anchor, engine, i, L, block, cos, sin, fault):
        unit = engine.layers[i]
        buf = engine.gather(unit)
        if i + 1 < len(engine.layers):
            engine.gather(engine.layers[i + 1], prefetch=True)
        layer = engine.model.text_model.layers[i]
        params, fused = engine.leaves(unit, buf, None)
        _bind(layer, fused)
        save = engine.save_cores and h.is_cuda
        try:
            if save:
                engine.act_store.gemms = engine.gemm_saved(i)
                engine.act_store.keep_act = engine.keep_act
                engine.act_store.begin("save", i)
            with nvtx(f"layer{i}.fwd"), torch.no_grad(), torch.nn.utils.stateless._reparametrize_module(layer, params):
                out = layer_step(layer, engine.cfg.layer_types[i], h, L, block, engine.cfg.gdn_chunk_size, cos, sin,
                                 fault)
        finally:
            if save:
                engine.act_store.end()
            _unbind(layer, fused)
        engine.check_gathered()
        ctx.save_for_backward(h, cos, sin)
        ctx.meta = (engine, i, L, block, fault)
        return out

    @staticmethod
    def backward(ctx, dout):
        h, cos, sin = ctx.saved_tensors
        engine, i, L, block, fault = ctx.meta
        unit = engine.layers[i]
        buf = engine.gather(unit)
        if i > 0:
            engine.gather(engine.layers[i - 1], prefetch=True)
        grad = engine.grad_buffer(unit)
        params, fused = engine.leaves(unit, buf, grad)
        layer = engine.model.text_model.layers[i]
        hx = h.detach().requires_grad_(True)
        _bind(layer, fused)
        reuse = engine.save_cores and hx.is_cuda
        try:
            if reuse:  # the recomputation takes the saved core outputs instead of rerunning them
                engine.act_store.gemms = engine.gemm_saved(i)
                engine.act_store.keep_act = engine.keep_act
                engine.act_store.begin("reuse", i)
            with nvtx(f"layer{i}.bwd"), torch.enable_grad(), \
                    torch.nn.utils.stateless._reparametrize_module(layer, params):
                out = layer_step(layer, engine.cfg.layer_types[i], hx, L, block, engine.cfg.gdn_chunk_size, cos, sin,
                                 fault)
                if reuse:
                    engine.act_store.end()
                torch.autograd.backward(out, dout)
        finally:
            if reuse:
                engine.act_store.end()
            _unbind(layer, fused)
        engine.check_gathered()
        engine.reduce_scatter(unit, grad)
        return hx.grad, None, None, None, None, None, None, None, None


def _head_loss(engine, ht, m, x0, norm_w, head_w, n_global, n_local):
    hn = ops.rmsnorm(ht, norm_w, engine.cfg.rms_norm_eps)
    if n_local == 0:
        # no scored target on this rank: a zero that still depends on the hidden states, so the
        # backward runs every layer and this rank joins every gather and reduce-scatter with zero
        # gradients (the reference's rule, `fsdp_train.py:618-629`)
        return hn.float().sum() * 0.0
    flat = m.reshape(-1)
    idx = torch.nonzero_static(flat, size=n_local).squeeze(1) if n_local is not None else flat.nonzero().squeeze(1)
    rows = hn.reshape(-1, hn.shape[-1]).index_select(0, idx)
    tgt = x0.reshape(-1).index_select(0, idx)
    return ops.masked_ce_sum(rows, head_w, tgt) / n_global


class _HeadFn(torch.autograd.Function):
    """final norm + masked-row lm_head + CE sum / global target count."""

    @staticmethod
    def forward(ctx, ht, m, x0, anchor, engine, n_global, n_local):
        u = engine.head
        buf = engine.gather(u)
        v = u.views(buf)
        if engine.tied:
            head_w = engine.embed.views(engine.gather(engine.embed))["weight"]
            buf = engine.gather(u)  # both resident: the two gathered slots hold head and embed
            v = u.views(buf)
        else:
            head_w = v["lm_head.weight"]
        ctx.meta = (engine, n_global, n_local)
        ctx.save_for_backward(ht, m, x0)
        with torch.no_grad():
            return _head_loss(engine, ht, m, x0, v["norm.weight"], head_w, n_global, n_local)

    @staticmethod
    def backward(ctx, g):
        engine, n_global, n_local = ctx.meta
        ht, m, x0 = ctx.saved_tensors
        engine.phase = "bwd"  # the head's backward opens the backward pass
        u = engine.head
        grad = engine.grad_buffer(u)
        buf = engine.gather(u)
        params, _ = engine.leaves(u, buf, grad)
        if engine.tied:
            ebuf = engine.gather(engine.embed)
            e = engine.embed.entries[0]
            tgrad = torch.zeros(e[1], dtype=ebuf.dtype, device=ebuf.device)
            head_w = ebuf[e[2] : e[2] + e[3]].view(e[1]).detach().requires_grad_(True)
            head_w.grad = tgrad
            buf = engine.gather(u)
            params, _ = engine.leaves(u, buf, grad)
        else:
            head_w = params["lm_head.weight"]
        hx = ht.detach().requires_grad_(True)
        with torch.enable_grad():
            loss = _head_loss(engine, hx, m, x0, params["norm.weight"], head_w, n_global, n_local)
        torch.autograd.backward(loss, g)
        engine.reduce_scatter(u, grad)
        if engine.tied:
            engine.table_grad[: tgrad.numel()].copy_(tgrad.reshape(-1).float())
        return hx.grad, None, None, None, None, None, None


class FSDPTrainer:
    """Public step API over the sharded engine, same call as `train.trainer.Trainer.step`."""

    def __init__(self, model, *, block: int, mask_id: int, lr: float = 1e-5, grad_clip: float = 1.0,
                 uniform_rows: bool = True, **_ignored):
        self.engine = FSDPEngine(model, lr=lr, grad_clip=grad_clip)
        self.block, self.mask_id = block, mask_id
        self.uniform_rows = uniform_rows
        self.gstep = 0
        self.world, self.rank = self.engine.world, self.engine.rank

    def step(self, x0, prompt_len, valid_len, n_targets: int | None = None, n_global=None):
        """x0 [b, L] this rank's rows (host or device); returns this rank's loss contribution.

        n_targets: this rank's scored-target count; n_global: the count over all ranks (host
        number), when the caller already has it. A rank with no scored target still runs the whole
        step (zero loss and zero gradients) so its collectives stay in step with the others; a
        step whose GLOBAL count is zero must be skipped by every rank (the caller's decision)."""
        self.gstep += 1
        if n_targets is None:
            n_targets = int((valid_len - prompt_len).clamp(min=0).sum())
        dev = self.engine.device
        x0 = x0.to(dev, non_blocking=True)
        prompt_len = prompt_len.to(dev, non_blocking=True)
        valid_len = valid_len.to(dev, non_blocking=True)
        if n_global is None:
            if self.world == 1 or self.uniform_rows:
                n_global = n_targets * self.world  # every rank scores the same count (no communication)
            else:
                n_global = torch.tensor(float(n_targets), device=dev)
                dist.all_reduce(n_global)
        if self.world == 1 and n_targets == 0:
            raise ValueError("a step with zero scored targets; skip it")
        return self.engine.step(x0, prompt_len, valid_len, block=self.block, mask_id=self.mask_id,
                                n_local=n_targets, n_global=n_global, gstep=self.gstep)
