"""Native block-diffusion decode engine: static caches, device-side commit, CUDA-graph steps.

The same decoding as `infer/cached.py` (and therefore the golden decoder's rule,
`src/dllm_qwen38/decode.py:53-97`), organised for the GPU:

  * caches live in preallocated buffers: per attention layer K/V [B, max_len, Hk, Dh] (bf16),
    per GDN layer the fp32 state [B, Hv, Dk, Dv] and the conv tail [B, K-1, conv_dim];
  * a block pass writes the block's K/V into cache rows [p0, p0 + T) and attends over rows
    [0, p0 + T) (`_C.attn_prefix`, key count read on the device), runs each GDN layer from the
    cached state (`_C.gdn_rows`) after the tail-aware conv (`_C.conv_tail`); a commit pass also
    writes the new state and conv tail in place;
  * a denoise step = block pass + lm_head GEMM + `_C.confidence` (softmax max / argmax per row)
    + `_C.commit` (threshold / sub-block / at-least-one rule for every batch row on the device);
    the host reads one int per row (positions still masked) per step;
  * with `graphs=True` the denoise step and the commit pass are each captured once into a CUDA
    graph (inputs are static buffers updated in place: ids, mask, positions, key count) and
    replayed, so a step is one graph launch.

Temperature sampling is not offered here (the device commit rule is the greedy one); use
`infer/cached.py` for temperature > 0.
"""

from __future__ import annotations

import torch

from ..config import FULL, LINEAR
from ..ops import _native
from ..ops import reference as ref
from .golden import DecodeTrace


class DecodeEngine:
    def __init__(self, model, batch: int, max_len: int, block: int, *, threshold: float = 0.9,
                 sub_block: int | None = None, graphs: bool = True):
        self.C = _native.require()
        from ..ops import cuda as Cu

        self.Cu = Cu
        cfg = model.config
        tm = model.text_model
        self.cfg, self.model = cfg, model
        self.dev = tm.embed_tokens.weight.device
        self.dt = tm.embed_tokens.weight.dtype
        if self.dev.type != "cuda" or self.dt != torch.bfloat16:
            raise ValueError("DecodeEngine needs a bf16 model on a CUDA device")
        if block > 32 or block % 2:
            raise ValueError("DecodeEngine: block must be even and <= 32")
        B, T = batch, block
        self.B, self.T, self.max_len = B, T, (max_len + T - 1) // T * T
        self.threshold, self.sub_block = float(threshold), int(sub_block or 0)
        self.graphs = graphs
        dev = self.dev
        self.layers = []
        for i, layer in enumerate(tm.layers):
            kind = cfg.layer_types[i]
            e = {"kind": kind, "ln1": layer.input_layernorm, "ln2": layer.post_attention_layernorm,
                 "w_gu": torch.cat([layer.mlp.gate_proj.weight, layer.mlp.up_proj.weight], 0).contiguous(),
                 "w_down": layer.mlp.down_proj.weight}
            if kind == LINEAR:
                m = layer.linear_attn
                e.update(m=m, w_in=torch.cat([m.in_proj_qkv.weight, m.in_proj_z.weight, m.in_proj_b.weight,
                                              m.in_proj_a.weight], 0).contiguous(),
                         conv_w=m.conv1d.weight[:, 0, :].float().contiguous(),
                         S=torch.zeros(B, m.num_v_heads, m.head_k_dim, m.head_v_dim, device=dev),
                         tail=torch.zeros(B, m.conv_kernel_size - 1, m.conv_dim, device=dev, dtype=self.dt))
            elif kind == FULL:
                m = layer.self_attn
                e.update(m=m, w_qkv=torch.cat([m.q_proj.weight, m.k_proj.weight, m.v_proj.weight], 0).contiguous(),
                         K=torch.zeros(B, self.max_len, m.num_kv_heads, m.head_dim, device=dev, dtype=self.dt),
                         V=torch.zeros(B, self.max_len, m.num_kv_heads, m.head_dim, device=dev, dtype=self.dt))
            else:
                raise ValueError(kind)
            self.layers.append(e)
        self.cos_t, self.sin_t = ref.rope_cos_sin(torch.arange(self.max_len), cfg.rotary_dim, cfg.rope_theta,
                                                  self.dt, dev)
        self.head = model.lm_head.weight
        # static step buffers
        self.ids = torch.zeros(B, T, dtype=torch.long, device=dev)
        self.masked = torch.zeros(B, T, dtype=torch.bool, device=dev)
        self.pos = torch.zeros(T, dtype=torch.long, device=dev)
        self.tk = torch.zeros(1, dtype=torch.int32, device=dev)
        self.conf = torch.zeros(B * T, dtype=torch.float32, device=dev)
        self.pick = torch.zeros(B * T, dtype=torch.long, device=dev)
        self.fw = torch.zeros(B, dtype=torch.int32, device=dev)
        self.left = torch.zeros(B, dtype=torch.int32, device=dev)
        self.mask_id_t = torch.full((), cfg.mask_id, dtype=torch.long, device=dev)
        self._g_step = self._g_commit = None
        self.length = 0

    # ------------------------------------------------------------------ passes
    def reset(self) -> None:
        for e in self.layers:
            if e["kind"] == LINEAR:
                e["S"].zero_()
                e["tail"].zero_()
        self.length = 0

    def _gdn(self, e, n, commit: bool):
        C, Cu, m = self.C, self.Cu, e["m"]
        B, T = self.B, self.T
        proj = Cu.gemm_nt(n, e["w_in"])
        raw, z, b, a = torch.split(proj.view(B, T, -1), [m.conv_dim, m.value_dim, m.num_v_heads, m.num_v_heads], -1)
        mixed = C.conv_tail(raw, e["tail"], e["conv_w"], commit)
        q, k, v = torch.split(mixed, [m.key_dim, m.key_dim, m.value_dim], dim=-1)
        q = q.view(B, T, m.num_k_heads, m.head_k_dim)
        k = k.view(B, T, m.num_k_heads, m.head_k_dim)
        v = v.view(B, T, m.num_v_heads, m.head_v_dim)
        g, beta = C.gdn_gates_fwd(a, b, m.A_log, m.dt_bias)
        (o,) = C.gdn_rows(q, k, v, g, beta, e["S"],
                          e["S"] if commit else None, T)
        y = Cu.gated_rmsnorm(o, z.reshape(B, T, m.num_v_heads, m.head_v_dim), m.norm.weight, m.norm.eps)
        return y.reshape(B * T, m.value_dim), m.out_proj.weight

    def _attn(self, e, n, cos, sin):
        C, Cu, m = self.C, self.Cu, e["m"]
        B, T = self.B, self.T
        Hq, Hk, Dh = m.num_heads, m.num_kv_heads, m.head_dim
        proj = Cu.gemm_nt(n, e["w_qkv"]).view(B, T, -1)
        qg, k, v = torch.split(proj, [2 * Hq * Dh, Hk * Dh, Hk * Dh], dim=-1)
        qg = qg.view(B, T, Hq, 2 * Dh)
        q, gate = qg[..., :Dh], qg[..., Dh:]
        q, k = Cu.qk_norm_rope(q, k.view(B, T, Hk, Dh), m.q_norm.weight, m.k_norm.weight, m.q_norm.eps, cos, sin)
        e["K"].index_copy_(1, self.pos, k)
        e["V"].index_copy_(1, self.pos, v.view(B, T, Hk, Dh))
        o = C.attn_prefix(q, e["K"], e["V"], 0, self.tk, Dh ** -0.5)
        o = o * torch.sigmoid(gate)
        return o.reshape(B * T, Hq * Dh), m.o_proj.weight

    def _block_pass(self, commit: bool) -> torch.Tensor:
        """Hidden states [B*T, D] after the final norm for the tokens in `ids` (masked -> [MASK])."""
        Cu = self.Cu
        tm = self.model.text_model
        ids = torch.where(self.masked, self.mask_id_t, self.ids)
        h = torch.nn.functional.embedding(ids.view(-1), tm.embed_tokens.weight)
        cos, sin = self.cos_t.index_select(0, self.pos), self.sin_t.index_select(0, self.pos)
        for e in self.layers:
            n = Cu.rmsnorm(h, e["ln1"].weight, e["ln1"].eps)
            if e["kind"] == LINEAR:
                y, w_o = self._gdn(e, n, commit)
            else:
                y, w_o = self._attn(e, n, cos, sin)
            h = Cu.gemm_nt(y, w_o, residual=h)
            x = Cu.rmsnorm(h, e["ln2"].weight, e["ln2"].eps)
            act, _ = Cu.gemm_swiglu(x, e["w_gu"], e["w_gu"].shape[0] // 2, store_gu=False)
            h = Cu.gemm_nt(act, e["w_down"], residual=h)
        return Cu.rmsnorm(h, tm.norm.weight, tm.norm.eps)

    def _step(self) -> None:
        hid = self._block_pass(commit=False)
        logits = self.Cu.gemm_nt(hid, self.head)
        self.C.confidence(logits, self.conf, self.pick)
        self.C.commit(self.conf, self.pick, self.masked, self.ids, self.threshold, self.sub_block, self.fw, self.left)

    def _commit(self) -> None:
        self._block_pass(commit=True)

    def _run(self, which: str) -> None:
        fn = self._step if which == "step" else self._commit
        if not self.graphs:
            fn()
            return
        attr = "_g_step" if which == "step" else "_g_commit"
        g = getattr(self, attr)
        if g is None:
            # warm up on a side stream (allocations, tensor maps), then capture
            s = torch.cuda.Stream(self.dev)
            s.wait_stream(torch.cuda.current_stream(self.dev))
            snap = self._snapshot()
            with torch.cuda.stream(s):
                fn()
            torch.cuda.current_stream(self.dev).wait_stream(s)
            self._restore(snap)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                fn()
            setattr(self, attr, g)
            self._restore(snap)
        g.replay()

    def _snapshot(self):
        """Everything a pass mutates, so warm-up and capture leave no trace."""
        keep = [self.ids, self.masked, self.fw, self.left]
        for e in self.layers:
            keep += [e["S"], e["tail"]] if e["kind"] == LINEAR else []
        return [(t, t.clone()) for t in keep]

    @staticmethod
    def _restore(snap) -> None:
        for t, c in snap:
            t.copy_(c)

    # ------------------------------------------------------------------ public API
    def _set_block(self, p0: int) -> None:
        self.pos.copy_(torch.arange(p0, p0 + self.T))
        self.tk.fill_(p0 + self.T)

    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> None:
        """Commit the prompt's whole blocks. prompt [B, n] (device)."""
        n_full = (prompt.shape[1] // self.T) * self.T
        self.masked.zero_()
        for p0 in range(0, n_full, self.T):
            self.ids.copy_(prompt[:, p0 : p0 + self.T])
            self._set_block(p0)
            self._run("commit")
        self.length = n_full

    @torch.no_grad()
    def generate(self, prompt_ids, *, n_blocks: int, eos_id: int | None = None) -> list:
        """Equal-length prompts (list of lists); returns one DecodeTrace per row."""
        rows = [list(p) for p in prompt_ids]
        if len(rows) != self.B or len({len(r) for r in rows}) != 1:
            raise ValueError(f"DecodeEngine was built for batch {self.B} of equal-length prompts")
        n = len(rows[0])
        if n + n_blocks * self.T > self.max_len:
            raise ValueError("prompt + generation exceed max_len")
        self.reset()
        cur = torch.tensor(rows, dtype=torch.long, device=self.dev)
        traces = [DecodeTrace(tokens=list(r)) for r in rows]
        self.prefill(cur)
        done = [False] * self.B
        T = self.T
        for _ in range(n_blocks):
            p0 = (n // T) * T
            k = n - p0
            blk = torch.full((self.B, T), self.cfg.mask_id, dtype=torch.long, device=self.dev)
            blk[:, :k] = cur[:, p0:n]
            self.ids.copy_(blk)
            msk = torch.zeros(self.B, T, dtype=torch.bool)
            msk[:, k:] = True
            for r in range(self.B):
                if done[r]:
                    msk[r] = False
            self.masked.copy_(msk)
            self.fw.zero_()
            self._set_block(p0)
            steps = 0
            while True:
                self._run("step")
                steps += 1
                if int(self.left.sum()) == 0:  # one small device->host read per step
                    break
            self._run("commit")
            fw = self.fw.tolist()
            new = self.ids[:, k:].tolist()
            cur = torch.cat([cur, self.ids[:, k:]], 1)
            n += T - k
            for r in range(self.B):
                if done[r]:
                    continue
                traces[r].forwards += fw[r]
                traces[r].tokens.extend(new[r])
                traces[r].generated += len(new[r])
                traces[r].steps_per_block.append(steps)
                if eos_id is not None and eos_id in new[r]:
                    done[r] = True
            if all(done):
                break
        return traces
