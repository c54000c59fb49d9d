"""Tensor-parallel block-diffusion decoding (TP = 1, 2, 4, 8 GPUs of one node). The reference
decodes on one device only (`src/dllm_qwen38/decode.py:35-99`); the commit rule is the same.

Layout (Megatron-style, with the residual stream sharded by rows between the layers):
  * GDN: q/k heads and v heads split evenly (Hk/world, Hv/world per rank), with their rows of
    in_proj (qkv | z | b | a), conv channels, A_log, dt_bias, cached state and conv tail;
    out_proj is row-parallel (its input columns split the same way);
  * attention: q heads split evenly; each rank keeps the kv heads its q heads read (kv heads are
    replicated when there are fewer kv heads than ranks); o_proj row-parallel;
  * MLP: gate/up rows split (column-parallel, SwiGLU in the GEMM epilogue), down row-parallel;
  * lm_head: vocabulary rows split; the embedding table is replicated.

Per step, with M = batch * block rows and rank r owning rows [r*M/W, (r+1)*M/W):
  column-parallel GEMMs read the gathered normalized rows from this rank's heap, waiting inside the
  GEMM's producer warp until every rank has pushed its rows (fused all-gather -> GEMM); row-parallel
  GEMMs store their fp32 partial rows straight into the owners' slots over NVLink from the
  epilogue (fused GEMM -> reduce-scatter); `tp_reduce_norm_push` then sums the partials with the
  residual, applies the next RMSNorm and pushes the normalized rows to every rank. The vocab-
  parallel confidence is merged in rank order on every rank, so the commit rule (csrc/decode.cu)
  runs replicated and every rank holds the same tokens. Counters that order the collectives live on
  the device, so each step is one CUDA-graph replay per rank.

Launch one process per GPU (torchrun); every rank builds the same model (same seed) and keeps its
shard.
"""

from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..config import FULL, LINEAR
from ..ops import _native
from ..ops import reference as ref
from .golden import DecodeTrace

EPI_BF16, EPI_F32, EPI_SWIGLU, EPI_PEER_F32 = 0, 1, 4, 5

TIMING = os.environ.get("BDLLM_TP_TIMING", "0") == "1"


def _timed(name):
    """Per-phase device time (CUDA events) when BDLLM_TP_TIMING=1 and graphs are off: a breakdown
    of where a step's time goes, read with `TPDecodeEngine.timing()`."""
    def deco(fn):
        def wrap(self, *a, **k):
            if not (TIMING and not self.graphs):
                return fn(self, *a, **k)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            r = fn(self, *a, **k)
            e1.record()
            self._events.append((name, e0, e1))
            return r
        return wrap
    return deco


class TPDecodeEngine:
    def __init__(self, model, batch: int, max_len: int, block: int, *, threshold: float = 0.9,
                 sub_block: int | None = None, graphs: bool = True, timeout_s: float | None = None):
        from ..ops import cuda as Cu
        from ..parallel.peer import SymmetricHeap

        self.C, self.Cu = _native.require(), Cu
        self.world, self.rank = (dist.get_world_size(), dist.get_rank()) if dist.is_initialized() else (1, 0)
        W, r = self.world, self.rank
        cfg = model.config
        tm = model.text_model
        self.cfg = cfg
        self.dev = tm.embed_tokens.weight.device
        self.dt = torch.bfloat16
        B, T = batch, block
        M = B * T
        if M % W or block > 32 or block % 2:
            raise ValueError("TP decode: batch*block divisible by the world, block even and <= 32")
        self.B, self.T, self.M, self.R = B, T, M, M // W
        self.max_len = (max_len + T - 1) // T * T
        self.threshold, self.sub_block, self.graphs = float(threshold), int(sub_block or 0), graphs
        self.timeout = float(timeout_s if timeout_s is not None else os.environ.get("BDLLM_PEER_TIMEOUT_S", "60"))
        D = cfg.hidden_size
        V = cfg.vocab_size
        if V % W or cfg.intermediate_size % W or cfg.num_attention_heads % W:
            raise ValueError("TP decode: vocab, FFN width and q heads must divide by the world size")
        dev = self.dev
        # ---------------------------------------------------------------- shards
        self.layers = []
        F = cfg.intermediate_size
        Fl = F // W
        for i, layer in enumerate(tm.layers):
            kind = cfg.layer_types[i]
            mlp = layer.mlp
            e = {"kind": kind,
                 "ln1": (1.0 + layer.input_layernorm.weight.float()).contiguous(),
                 "ln2": (1.0 + layer.post_attention_layernorm.weight.float()).contiguous(),
                 "eps": layer.input_layernorm.eps,
                 "w_gu": torch.cat([mlp.gate_proj.weight[r * Fl:(r + 1) * Fl],
                                    mlp.up_proj.weight[r * Fl:(r + 1) * Fl]], 0).contiguous(),
                 "w_down": mlp.down_proj.weight[:, r * Fl:(r + 1) * Fl].contiguous()}
            if kind == LINEAR:
                m = layer.linear_attn
                Hk, Hv, Dk, Dv = m.num_k_heads, m.num_v_heads, m.head_k_dim, m.head_v_dim
                if Hk % W or Hv % W:
                    raise ValueError("TP decode: GDN heads must divide by the world size")
                hk, hv = Hk // W, Hv // W
                kd = m.key_dim
                qkv = m.in_proj_qkv.weight
                rows_q = slice(r * hk * Dk, (r + 1) * hk * Dk)
                rows_k = slice(kd + r * hk * Dk, kd + (r + 1) * hk * Dk)
                rows_v = slice(2 * kd + r * hv * Dv, 2 * kd + (r + 1) * hv * Dv)
                cw = m.conv1d.weight[:, 0, :]
                e.update(hk=hk, hv=hv, Dk=Dk, Dv=Dv,
                         w_in=torch.cat([qkv[rows_q], qkv[rows_k], qkv[rows_v],
                                         m.in_proj_z.weight[r * hv * Dv:(r + 1) * hv * Dv],
                                         m.in_proj_b.weight[r * hv:(r + 1) * hv],
                                         m.in_proj_a.weight[r * hv:(r + 1) * hv]], 0).contiguous(),
                         conv_w=torch.cat([cw[rows_q], cw[rows_k], cw[rows_v]], 0).float().contiguous(),
                         A_log=m.A_log[r * hv:(r + 1) * hv].detach().clone(),
                         dt_bias=m.dt_bias[r * hv:(r + 1) * hv].detach().clone(),
                         norm_w=m.norm.weight.detach().clone(), norm_eps=m.norm.eps,
                         w_out=m.out_proj.weight[:, r * hv * Dv:(r + 1) * hv * Dv].contiguous(),
                         S=torch.zeros(B, hv, Dk, Dv, device=dev),
                         tail=torch.zeros(B, m.conv_kernel_size - 1, 2 * hk * Dk + hv * Dv, device=dev, dtype=self.dt))
            elif kind == FULL:
                m = layer.self_attn
                Hq, Hk, Dh = m.num_heads, m.num_kv_heads, m.head_dim
                hq, grp = Hq // W, Hq // Hk
                kv0, kv1 = (r * hq) // grp, ((r + 1) * hq - 1) // grp + 1
                if hq % (kv1 - kv0):
                    raise ValueError("TP decode: local q heads must split evenly over the local kv heads")
                e.update(qn=m.q_norm.weight.detach().clone(), kn=m.k_norm.weight.detach().clone(), qk_eps=m.q_norm.eps,
                         hq=hq, hk=kv1 - kv0, Dh=Dh,
                         w_qkv=torch.cat([m.q_proj.weight[r * hq * 2 * Dh:(r + 1) * hq * 2 * Dh],
                                          m.k_proj.weight[kv0 * Dh:kv1 * Dh],
                                          m.v_proj.weight[kv0 * Dh:kv1 * Dh]], 0).contiguous(),
                         w_o=m.o_proj.weight[:, r * hq * Dh:(r + 1) * hq * Dh].contiguous(),
                         K=torch.zeros(B, self.max_len, kv1 - kv0, Dh, device=dev, dtype=self.dt),
                         V=torch.zeros(B, self.max_len, kv1 - kv0, Dh, device=dev, dtype=self.dt))
            else:
                raise ValueError(kind)
            self.layers.append(e)
        self.final_w1 = (1.0 + tm.norm.weight.float()).contiguous()
        self.final_eps = tm.norm.eps
        self.embed = tm.embed_tokens.weight.detach()
        self.Vl = V // W
        self.head = model.lm_head.weight[r * self.Vl:(r + 1) * self.Vl].contiguous()
        self.cos_t, self.sin_t = ref.rope_cos_sin(torch.arange(self.max_len), cfg.rotary_dim, cfg.rope_theta,
                                                  self.dt, dev)
        # ---------------------------------------------------------------- peer heap
        self.SMAX = 8
        self.n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        self._nslots = W
        part_bytes = W * self.SMAX * self.R * D * 4
        gather_bytes = M * D * 2
        conf_bytes = W * M * 16
        if W > 1:
            self.heap = SymmetricHeap(part_bytes + gather_bytes + conf_bytes + 3 * 256, dev)
            self.part, self.part_off = self.heap.alloc(W * self.SMAX * self.R * D, torch.float32)
            self.gather, self.gather_off = self.heap.alloc(M * D, self.dt)
            _, self.conf_off = self.heap.alloc(W * M * 4, torch.float32)
            self.peers = self.heap.ptrs
        else:
            self.heap = None
        self.part2d = self.part[: M * D].view(M, D) if W > 1 else None  # shape/stride template of the slots
        self.gather2d = self.gather.view(M, D) if W > 1 else None
        self.ctr = torch.zeros(16, dtype=torch.int32, device=dev)
        # ---------------------------------------------------------------- step buffers
        self.h = torch.zeros(self.R, D, dtype=self.dt, device=dev)
        self.ids = torch.zeros(B, T, dtype=torch.long, device=dev)
        self.masked = torch.zeros(B, T, dtype=torch.bool, device=dev)
        self.pos = torch.zeros(T, dtype=torch.long, device=dev)
        self.tk = torch.zeros(1, dtype=torch.int32, device=dev)
        self.conf = torch.zeros(M, dtype=torch.float32, device=dev)
        self.pick = torch.zeros(M, dtype=torch.long, device=dev)
        self.fw = torch.zeros(B, dtype=torch.int32, device=dev)
        self.left = torch.zeros(B, dtype=torch.int32, device=dev)
        self.mask_id_t = torch.full((), cfg.mask_id, dtype=torch.long, device=dev)
        self._g = {}
        self._events = []
        if W > 1:
            torch.cuda.synchronize(dev)
            dist.barrier()

    # ------------------------------------------------------------------ collectives
    def _splits(self, N: int, K: int) -> int:
        """k-splits so that a skinny GEMM (few output tiles) still runs one wave over the SMs."""
        if self.M > 256 or N % 8 or K < 1024:
            return 1
        tiles = ((self.M + 127) // 128) * ((N + 255) // 256)
        return max(1, min(self.SMAX, self.n_sms // tiles, K // 64 // 2))

    @_timed("col_gemm")
    def _col(self, w, epi=EPI_BF16):
        """Column-parallel GEMM over the gathered rows (waits for every rank's push inside the GEMM)."""
        C = self.C
        N = w.shape[0] // 2 if epi == EPI_SWIGLU else w.shape[0]
        if self.world == 1:
            if epi == EPI_SWIGLU:
                return self.Cu.gemm_swiglu(self._a1, w, N, store_gu=False)[0]
            return self.Cu.gemm_nt(self._a1, w)
        S = self._splits(w.shape[0], w.shape[1])
        if S > 1:  # fp32 k-split partials, then one reduction (SwiGLU applied there)
            ws = torch.empty(S * self.M * w.shape[0], dtype=torch.float32, device=self.dev)
            S = C.gemm_tp(self.gather2d, w, ws.view(-1, w.shape[0]), EPI_F32, None, self.peers, self.rank, self.R,
                          self.part_off, 0, self.ctr, True, self.timeout, 256, S)
            out = torch.empty(self.M, N, dtype=self.dt, device=self.dev)
            C.splitk_reduce(ws, S, out, None, epi == EPI_SWIGLU)
            self.Cu._count(2)
            return out
        pad = -(-N // 8) * 8  # 16-byte output rows
        out = torch.empty(self.M, pad, dtype=self.dt, device=self.dev)[:, :N]
        C.gemm_tp(self.gather2d, w, out, epi, None, self.peers, self.rank, self.R, self.part_off, 0, self.ctr, True,
                  self.timeout, 256, 1)
        self.Cu._count()
        return out

    @_timed("row_gemm")
    def _row(self, x, w):
        """Row-parallel GEMM: fp32 partial rows straight into the owners' slots (per k split)."""
        if self.world == 1:
            self._partial = self.Cu.gemm_nt(x, w)
            return
        S = self._splits(w.shape[0], w.shape[1])
        self._nslots = self.world * self.C.gemm_tp(x, w, self.part2d, EPI_PEER_F32, None, self.peers, self.rank,
                                                   self.R, self.part_off, 0, self.ctr, False, self.timeout, 256, S)
        self.Cu._count()

    @_timed("reduce_norm_push")
    def _reduce_norm(self, w1, eps, has_partials=True, push=True):
        if self.world == 1:
            if has_partials:
                self.h.copy_((self._partial.float() + self.h.float()).to(self.dt))
            if push:
                self._a1 = self.C.rmsnorm_fwd(self.h, w1, eps)
            return
        self.C.tp_reduce_norm_push(self.peers, self.rank, self.R, self.cfg.hidden_size, self.part_off, self.h,
                                   has_partials, w1, eps, self.gather_off, 0, self.ctr, self.timeout, push,
                                   self._nslots if has_partials else 0)
        self.Cu._count()

    # ------------------------------------------------------------------ mixers (local heads, all M rows)
    @_timed("gdn_mixer_total")
    def _gdn(self, e, commit):
        C, Cu, B, T = self.C, self.Cu, self.B, self.T
        hk, hv, Dk, Dv = e["hk"], e["hv"], e["Dk"], e["Dv"]
        proj = self._col(e["w_in"]).view(B, T, -1)
        cd = 2 * hk * Dk + hv * Dv
        raw, z, b, a = torch.split(proj, [cd, hv * Dv, hv, hv], -1)
        mixed = C.conv_tail(raw, e["tail"], e["conv_w"], commit)
        q, k, v = torch.split(mixed, [hk * Dk, hk * Dk, hv * Dv], dim=-1)
        g, beta = C.gdn_gates_fwd(a, b, e["A_log"], e["dt_bias"])
        (o,) = C.gdn_rows(q.view(B, T, hk, Dk), k.view(B, T, hk, Dk), v.view(B, T, hv, Dv), g.float().contiguous(),
                          beta.float().contiguous(), e["S"], e["S"] if commit else None, T)
        y = Cu.gated_rmsnorm(o, z.reshape(B, T, hv, Dv), e["norm_w"], e["norm_eps"])
        self._row(y.reshape(B * T, hv * Dv), e["w_out"])

    @_timed("attn_mixer_total")
    def _attn(self, e, cos, sin):
        C, Cu, B, T = self.C, self.Cu, self.B, self.T
        hq, hk, Dh = e["hq"], e["hk"], e["Dh"]
        proj = self._col(e["w_qkv"]).view(B, T, -1)
        qg, k, v = torch.split(proj, [2 * hq * Dh, hk * Dh, hk * Dh], dim=-1)
        qg = qg.view(B, T, hq, 2 * Dh)
        q, gate = qg[..., :Dh], qg[..., Dh:]
        q, k = Cu.qk_norm_rope(q, k.view(B, T, hk, Dh), e["qn"], e["kn"], e["qk_eps"], cos, sin)
        e["K"].index_copy_(1, self.pos, k)
        e["V"].index_copy_(1, self.pos, v.view(B, T, hk, Dh))
        o = C.attn_prefix(q, e["K"], e["V"], 0, self.tk, Dh ** -0.5) * torch.sigmoid(gate)
        self._row(o.reshape(B * T, hq * Dh), e["w_o"])

    def _block_pass(self, commit: bool) -> None:
        ids = torch.where(self.masked, self.mask_id_t, self.ids).view(-1)[self.rank * self.R:(self.rank + 1) * self.R]
        self.h.copy_(torch.nn.functional.embedding(ids, self.embed))
        cos, sin = self.cos_t.index_select(0, self.pos), self.sin_t.index_select(0, self.pos)
        L = self.layers
        self._reduce_norm(L[0]["ln1"], L[0]["eps"], has_partials=False)
        for i, e in enumerate(L):
            if e["kind"] == LINEAR:
                self._gdn(e, commit)
            else:
                self._attn(e, cos, sin)
            self._reduce_norm(e["ln2"], e["eps"])
            act = self._col(e["w_gu"], EPI_SWIGLU)
            self._row(act, e["w_down"])
            last = i + 1 == len(L)
            if last:
                self._reduce_norm(self.final_w1, self.final_eps, push=not commit)
            else:
                self._reduce_norm(L[i + 1]["ln1"], L[i + 1]["eps"])

    def _step(self) -> None:
        self._block_pass(commit=False)
        logits = self._col(self.head)
        if self.world == 1:
            self.C.confidence(logits, self.conf, self.pick)
        else:
            self.C.tp_confidence(self.peers, self.rank, logits, self.rank * self.Vl, self.conf_off, 0, self.ctr,
                                 self.conf, self.pick, self.timeout)
            self.Cu._count(2)
        self.C.commit(self.conf, self.pick, self.masked, self.ids, self.threshold, self.sub_block, self.fw, self.left)

    def _commit(self) -> None:
        self._block_pass(commit=True)

    def _run(self, which: str) -> None:
        fn = self._step if which == "step" else self._commit
        if not self.graphs:
            fn()
            return
        g = self._g.get(which)
        if g is None:
            # warm-up (tensor maps, allocator) then capture; both leave the caches as they were and
            # keep the device counters in step with the peers (every rank does the same passes)
            snap = self._snapshot()
            fn()
            torch.cuda.synchronize(self.dev)
            self._restore(snap)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            self._g[which] = g
            self._restore(snap)
        g.replay()

    def _snapshot(self):
        keep = [self.ids, self.masked, self.fw, self.left, self.h]
        for e in self.layers:
            keep += [e["S"], e["tail"]] if e["kind"] == LINEAR else []
        return [(t, t.clone()) for t in keep]

    @staticmethod
    def _restore(snap) -> None:
        for t, c in snap:
            t.copy_(c)

    # ------------------------------------------------------------------ public API
    def reset(self) -> None:
        for e in self.layers:
            if e["kind"] == LINEAR:
                e["S"].zero_()
                e["tail"].zero_()

    def _set_block(self, p0: int) -> None:
        self.pos.copy_(torch.arange(p0, p0 + self.T))
        self.tk.fill_(p0 + self.T)

    @torch.no_grad()
    def generate(self, prompt_ids, *, n_blocks: int, eos_id: int | None = None) -> list:
        """Equal-length prompts (the same on every rank); returns one DecodeTrace per row."""
        rows = [list(p) for p in prompt_ids]
        if len(rows) != self.B or len({len(x) for x in rows}) != 1:
            raise ValueError(f"TPDecodeEngine was built for batch {self.B} of equal-length prompts")
        n = len(rows[0])
        if n + n_blocks * self.T > self.max_len:
            raise ValueError("prompt + generation exceed max_len")
        self.reset()
        T = self.T
        cur = torch.tensor(rows, dtype=torch.long, device=self.dev)
        traces = [DecodeTrace(tokens=list(x)) for x in rows]
        self.masked.zero_()
        for p0 in range(0, (n // T) * T, T):
            self.ids.copy_(cur[:, p0:p0 + T])
            self._set_block(p0)
            self._run("commit")
        done = [False] * self.B
        for _ in range(n_blocks):
            p0 = (n // T) * T
            k = n - p0
            blk = torch.full((self.B, T), self.cfg.mask_id, dtype=torch.long, device=self.dev)
            blk[:, :k] = cur[:, p0:n]
            self.ids.copy_(blk)
            msk = torch.zeros(self.B, T, dtype=torch.bool)
            msk[:, k:] = True
            for i in range(self.B):
                if done[i]:
                    msk[i] = False
            self.masked.copy_(msk)
            self.fw.zero_()
            self._set_block(p0)
            steps = 0
            while True:
                self._run("step")
                steps += 1
                if int(self.left.sum()) == 0:
                    break
            self._run("commit")
            fw = self.fw.tolist()
            new = self.ids[:, k:].tolist()
            cur = torch.cat([cur, self.ids[:, k:]], 1)
            n += T - k
            for i in range(self.B):
                if done[i]:
                    continue
                traces[i].forwards += fw[i]
                traces[i].tokens.extend(new[i])
                traces[i].generated += len(new[i])
                traces[i].steps_per_block.append(steps)
                if eos_id is not None and eos_id in new[i]:
                    done[i] = True
            if all(done):
                break
        return traces

    def timing(self) -> dict:
        """{phase: total ms} of the timed calls so far (BDLLM_TP_TIMING=1, graphs off)."""
        torch.cuda.synchronize(self.dev)
        out = {}
        for name, e0, e1 in self._events:
            out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
        return {k: round(v, 2) for k, v in out.items()}

    def close(self) -> None:
        self._g.clear()
        if self.heap is not None:
            torch.cuda.synchronize(self.dev)
            dist.barrier()
            self.heap.close()
            self.heap = None
