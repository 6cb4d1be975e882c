"""OneSdmLM (the PARTIAL `onesdm` and FULL `onesdm_allsdm` arms) on libsdm_b200, plus a carried-state decoder.

Mirrors track4_onesdm_models.py:471-564 (OneSdmLM), :591-633 (DEFAULTS, lm_kwargs, allsdm_n_sub, build_onesdm):
same constructor, module tree, parameter names, init order and state_dict keys.  The forward runs layer by layer
through the C ABI with every residual add fused into the producing GEMM's epilogue.  The Archive (off by default
in the reference) and the transformer/sdmonly comparison arms are not part of this path and raise.

The decode API is new (the reference has no carried-state decode): `prefill` runs the chunked prefill and keeps
each layer's final memory state, `decode_step` advances every stream by one token reading and writing that state in
place, and `generate` does greedy decoding.
"""
import math

import torch
import torch.nn as nn

from ._lib import check, lib, ptr, stream_ptr, workspace, dtype_code
from .modules import RMSNorm, RunTimeSdm, SwiGLU, TrainedSdm, matched_sdm_n_sub, _forward_only


class OneSdmLM(nn.Module):
    kind = "onesdm"

    def __init__(self, V, d=256, layers=4, mlp_f=688, mem=True, heads=4, n_sub=32, d_a=32, k=16,
                 decays=(0.0, 0.8, 0.99, 1.0), learn_decay=False, write_gate=True, gate_bias=0.0, read_mode="mean",
                 out_norm=True, addr_scale=8.0, learn_scale=True, chunk=128, mem_in_grad=1.0, out_norm_eps=1e-2,
                 read_eps=1e-3, addr_bias=0.0, archive=False,
                 arc_layers=None, arc_d_c=64, arc_n_sub=16, arc_k=4, arc_slot_keep=4, arc_window=16, arc_n_fetch=4,
                 arc_weighting="soft", tie=True, ffn="mlp", sdm_n_sub=0, sdm_heads=4, sdm_d_a=0, sdm_k=32,
                 sdm_scale=8.0, sdm_learn_scale=True, reset_at_bos=False, bos_id=0, seed=0):
        super().__init__()
        assert ffn in ("mlp", "sdm", "none")
        if archive:
            raise NotImplementedError("the Archive (pointer SDM, off by default in the reference) is not on this path")
        if not tie:
            raise NotImplementedError("the untied head is not on this path (the PARTIAL and FULL arms tie)")
        self.V, self.d, self.n_layers, self.mlp_f, self.tie = V, d, layers, mlp_f, tie
        self.reset_at_bos, self.bos_id = reset_at_bos, bos_id
        self.ffn = ffn
        self.has_mem, self.has_arc = mem, False
        self.emb = nn.Embedding(V, d)
        self.mems = nn.ModuleList([RunTimeSdm(d, heads, n_sub, d_a, k, tuple(decays), learn_decay, write_gate,
                                              gate_bias, read_mode, out_norm, addr_scale, learn_scale, chunk,
                                              read_eps=read_eps, mem_in_grad=mem_in_grad, out_norm_eps=out_norm_eps,
                                              addr_bias=addr_bias, seed=seed + 31 * i) for i in range(layers)])
        for m in self.mems:
            m.enabled = mem
        self.arc_layers = tuple(range(1, layers)) if arc_layers is None else tuple(arc_layers)
        if ffn == "mlp":
            self.mnorms = nn.ModuleList([RMSNorm(d) for _ in range(layers)])
            self.mlps = nn.ModuleList([SwiGLU(d, mlp_f) for _ in range(layers)])
        elif ffn == "sdm":
            self.sdm_d_a = sdm_d_a or min(32, (d // sdm_heads) // 2 * 2)
            self.sdm_n_sub = sdm_n_sub or matched_sdm_n_sub(d, mlp_f, sdm_heads, self.sdm_d_a)
            self.sdms = nn.ModuleList([TrainedSdm(d, self.sdm_n_sub, sdm_heads, self.sdm_d_a, sdm_k, sdm_scale,
                                                  sdm_learn_scale, seed=seed + 53 * i) for i in range(layers)])
        self.nf = RMSNorm(d)
        nn.init.normal_(self.emb.weight, std=0.02)
        for n, p in self.named_parameters():
            if p.dim() == 2 and "emb" not in n and "onorm_w" not in n and "addr_b" not in n:
                out_map = n.endswith("down.weight") or (n.startswith("sdms.") and n.endswith("wo.weight"))
                nn.init.normal_(p, std=0.02 / math.sqrt(2 * layers) if out_map else 0.02)
        for m in self.mems:
            m.reset_init()
        for s in getattr(self, "sdms", []):
            s.reset_init()

    # ------------------------------------------------------------------------------------------ precision
    def to_bf16_stream(self):
        """bfloat16 token table, norms and matrices (the tensor-core path); sub-keys, address biases, scales,
        fades, out-norm weights and the gate bias stay float32."""
        keep32 = ("keys1", "keys2", "addr_b", "log_scale", "decay_logit", "onorm_w", "wg.bias")
        for n, p in self.named_parameters():
            if not any(n.endswith(s) for s in keep32):
                p.data = p.data.to(torch.bfloat16)
        return self

    @property
    def stream_dtype(self):
        return self.emb.weight.dtype

    # ------------------------------------------------------------------------------------------ forward
    def enfold(self, idx):
        """OneSdmLM.enfold (M:525-526): the token table lookup."""
        ids = idx.to(torch.int32).contiguous()
        N = ids.numel()
        E = self.emb.weight
        out = torch.empty(*idx.shape, self.d, dtype=E.dtype, device=E.device)
        bad = torch.zeros(1, dtype=torch.int32, device=E.device)
        check(lib().sdm_embed(ptr(ids), ptr(E.detach()), N, self.d, self.V, dtype_code(E.dtype), ptr(out), ptr(bad),
                              stream_ptr(E.device)), "sdm_embed")
        return out, bad

    def residual(self, idx, sequential=False, trace=None):
        """OneSdmLM.residual (M:534-548) with each residual add fused into the module's last GEMM.  trace: a list
        that receives, per layer, the layer input, the stream after the memory, the memory's addresses z
        (B, T, 2, h, d_a) and slot ids (write and read, (B, h, T, k)), and the TrainedSdm queries (B*T, h, d_a) and
        slot ids (B*T, h, k)."""
        _forward_only(self.emb.weight)
        x, _ = self.enfold(idx)
        reset = (idx == self.bos_id) if self.reset_at_bos else None
        for i in range(self.n_layers):
            x = self._layer(i, x, reset, sequential, trace)
        return x

    def _layer(self, i, x, reset, sequential=False, trace=None):
        """Layer i of residual(): the memory, then the body, each with its residual add."""
        m = self.mems[i]
        rec = None if trace is None else {"x_in": x}
        if m.enabled:
            if sequential:
                x = x + m.forward_sequential(x, reset)
            elif rec is not None:
                x, o = m._run(x, reset, add_residual=True, want=("sel", "z"))
                rec["siw"], rec["sir"], rec["z"] = o["siw"], o["sir"], o["z"]
            else:
                x = m._run(x, reset, add_residual=True)[0]
        if rec is not None:
            rec["x_mid"] = x
        if self.ffn == "mlp":
            x = self.mlps[i].block(x, self.mnorms[i].w, self.mnorms[i].eps)
        elif self.ffn == "sdm":
            if rec is not None:
                x, rec["sdm_si"], _, rec["sdm_q"] = self.sdms[i]._run(x, add_residual=True, want_sel=True, want_q=True)
            else:
                x = self.sdms[i]._run(x, add_residual=True)[0]
        if rec is not None:
            trace.append(rec)
        return x

    def hidden(self, idx, sequential=False):
        return self.nf(self.residual(idx, sequential))

    def project(self, h):
        """OneSdmLM.project (M:528-529): the tied head h @ E^T (no norm), in h's dtype, on the library's GEMM."""
        _forward_only(h, self.emb.weight)
        h = h.contiguous()
        E = self.emb.weight.detach().to(h.dtype).contiguous()
        out = torch.empty(*h.shape[:-1], self.V, dtype=h.dtype, device=h.device)
        check(lib().sdm_tied_project(ptr(h), ptr(E), h.numel() // self.d, self.d, self.V, dtype_code(h.dtype), ptr(out),
                                     stream_ptr(h.device)), "sdm_tied_project")
        return out

    def unfold(self, x):
        return self.project(self.nf(x))

    def _head(self, x, mode, targets=None, out=None):
        x = x.contiguous()
        N = x.numel() // self.d
        dt = x.dtype
        ws = workspace(lib().sdm_tied_head_workspace_size(N, self.d, self.V, dtype_code(dt)), x.device)
        E = self.emb.weight.detach()
        nfw = self.nf.w.detach().to(dt).contiguous()
        st = stream_ptr(x.device)
        if mode == "logits":
            out = torch.empty(*x.shape[:-1], self.V, dtype=dt, device=x.device)
            check(lib().sdm_tied_logits(ptr(x), ptr(nfw), ptr(E), N, self.d, self.V, self.nf.eps, dtype_code(dt),
                                        ptr(out), ptr(ws), ws.numel(), st), "sdm_tied_logits")
            return out
        if mode == "ce":
            tg = targets.to(torch.int32).contiguous()
            out = torch.zeros(1, dtype=torch.float64, device=x.device) if out is None else out
            check(lib().sdm_tied_ce_sum(ptr(x), ptr(nfw), ptr(E), ptr(tg), N, self.d, self.V, self.nf.eps,
                                        dtype_code(dt), ptr(out), ptr(ws), ws.numel(), st), "sdm_tied_ce_sum")
            return out
        ids = torch.empty(x.shape[:-1], dtype=torch.int32, device=x.device)
        check(lib().sdm_tied_argmax(ptr(x), ptr(nfw), ptr(E), N, self.d, self.V, self.nf.eps, dtype_code(dt),
                                    ptr(ids), ptr(ws), ws.numel(), st), "sdm_tied_argmax")
        return ids

    def forward(self, idx, sequential=False):
        """OneSdmLM.forward (M:554-555): logits (B, T, V) = nf(residual(idx)) @ E^T, in the stream dtype."""
        return self._head(self.residual(idx, sequential), "logits")

    def loss_sum(self, idx, targets, out=None, row_streams=1):
        """Sum over positions of the tied-head cross-entropy against `targets` (B, T) (entries < 0 skipped), as a
        float64 device scalar accumulated into `out` if given; the logits are never materialised whole.

        row_streams > 1 splits the rows (independent sequences) into that many groups, each run on its own CUDA
        stream after the current one, so one group's kernels fill the other's partial waves; the work is submitted
        layer by layer across the groups (so every stream has queued work from the start) and the current stream
        waits for all of them.  The sum is the same up to the order of its float64 additions."""
        B = idx.shape[0]
        if row_streams <= 1 or B < row_streams:
            return self._head(self.residual(idx), "ce", targets, out)
        if out is None:
            out = torch.zeros(1, dtype=torch.float64, device=idx.device)
        main = torch.cuda.current_stream(idx.device)
        key = (idx.device.index, row_streams)
        cache = self.__dict__.setdefault("_row_stream_cache", {})
        if key not in cache:  # created once: a new stream per call would cost host time and hardware queues
            cache[key] = [torch.cuda.Stream(idx.device) for _ in range(row_streams)]
        side = cache[key]
        bounds = [B * i // row_streams for i in range(row_streams + 1)]
        for s in side:
            s.wait_stream(main)
        _forward_only(self.emb.weight)
        xs, resets = [], []
        for s, r0, r1 in zip(side, bounds[:-1], bounds[1:]):
            with torch.cuda.stream(s):
                xs.append(self.enfold(idx[r0:r1])[0])
                resets.append((idx[r0:r1] == self.bos_id) if self.reset_at_bos else None)
        for i in range(self.n_layers):
            for g, s in enumerate(side):
                with torch.cuda.stream(s):
                    xs[g] = self._layer(i, xs[g], resets[g])
        for g, (s, r0, r1) in enumerate(zip(side, bounds[:-1], bounds[1:])):
            with torch.cuda.stream(s):
                self._head(xs[g], "ce", targets[r0:r1], out)
        for s in side:
            main.wait_stream(s)
        return out

    def loss_graph(self, B, T, row_streams=1, device=None):
        """Capture loss_sum over a (B, T) batch as one CUDA graph; returns step(idx, targets) -> the (1,) float64
        device loss sum (the graph's static output, overwritten by the next call).

        The step launches about a dozen kernels per layer; replaying them as a graph removes the host's per-launch
        work, which at a few rows per GPU is as long as the kernels themselves.  idx and targets (B, T) may be host
        tensors (pinned memory copies asynchronously) or device tensors; they are copied into static buffers.  Warm-up
        runs on a side stream before capture, so every weight cache and workspace exists when the graph is built."""
        dev = device or self.emb.weight.device
        ids_in = torch.zeros(B, T, dtype=torch.int32, device=dev)
        tgt_in = torch.full((B, T), -1, dtype=torch.int32, device=dev)
        out = torch.zeros(1, dtype=torch.float64, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(2):
                self.loss_sum(ids_in, tgt_in, out=out, row_streams=row_streams)
        torch.cuda.current_stream(dev).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph), torch.no_grad():
            out.zero_()
            self.loss_sum(ids_in, tgt_in, out=out, row_streams=row_streams)

        def step(idx, targets):
            ids_in.copy_(idx, non_blocking=True)
            tgt_in.copy_(targets, non_blocking=True)
            graph.replay()
            return out
        step.graph = graph
        return step

    def memory_parameters(self):
        return {n for n, _ in self.named_parameters() if n.startswith("mems.")}

    def set_leak(self, on):
        """OneSdmLM.set_leak (M:560-564): the reference's test-only causality-leak switch of every memory.  The
        kernels have no leaking variant, so a forward with the switch on raises NotImplementedError."""
        for m in self.mems:
            m._leak = on

    # ------------------------------------------------------------------------------------------ decode
    def init_decode(self, S, device=None):
        """Empty carried state for S streams: one dict per layer (see RunTimeSdm.init_state)."""
        device = device or self.emb.weight.device
        return [m.init_state(S, device) for m in self.mems]

    def prefill(self, idx, state):
        """Run the prompt idx (S, T) through the chunked path, leave each layer's final memory in `state`, and
        return the greedy next token of every stream (S,) int32."""
        _forward_only(self.emb.weight)
        x, _ = self.enfold(idx)
        reset = (idx == self.bos_id) if self.reset_at_bos else None
        for i in range(self.n_layers):
            m, st = self.mems[i], state[i]
            if m.enabled:
                x, o = m._run(x, reset, add_residual=True, want=("sel",))
                st["mem"].copy_(m.last_state[0])
                st["cnt"].copy_(m.last_state[1])
                st["scale"].fill_(1.0)
                st["last_w"].copy_(o["siw"][:, :, -1, :])
            if self.ffn == "mlp":
                x = self.mlps[i].block(x, self.mnorms[i].w, self.mnorms[i].eps)
            elif self.ffn == "sdm":
                x = self.sdms[i]._run(x, add_residual=True)[0]
        return self._head(x[:, -1], "argmax")

    def decode_step(self, ids, state, reset=None):
        """Advance every stream by one token ids (S,): all layers read and write their carried state in place.
        Returns the greedy next token (S,) int32."""
        _forward_only(self.emb.weight)
        x, _ = self.enfold(ids)
        if reset is None and self.reset_at_bos:
            reset = ids == self.bos_id
        for i in range(self.n_layers):
            m = self.mems[i]
            if m.enabled:
                x = m.decode_step(x, state[i], reset, add_residual=True)
            if self.ffn == "mlp":
                x = self.mlps[i].block(x, self.mnorms[i].w, self.mnorms[i].eps)
            elif self.ffn == "sdm":
                x = self.sdms[i]._run(x, add_residual=True)[0]
        return self._head(x, "argmax")

    def decode_graph(self, state):
        """Capture one decode_step over `state` (all its streams) as a CUDA graph; returns step(ids) -> next ids.

        The graph replays every kernel of the step with no host work in between (the step is otherwise bound by
        ~100 launches and their Python/ctypes overhead).  Inputs are copied into a static buffer; the returned ids
        tensor is the graph's static output (overwritten by the next call).  Warm-up runs on a saved copy of the
        state, which is restored before capture, so building the graph does not advance any stream."""
        S = state[0]["mem"].shape[0]
        dev = state[0]["mem"].device
        ids_in = torch.zeros(S, dtype=torch.int64, device=dev)
        saved = [{k: v.clone() for k, v in st.items()} for st in state]
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(2):
                self.decode_step(ids_in, state)
        torch.cuda.current_stream(dev).wait_stream(side)
        for st, sv in zip(state, saved):
            for k in st:
                st[k].copy_(sv[k])
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph), torch.no_grad():
            ids_out = self.decode_step(ids_in, state)

        def step(ids):
            ids_in.copy_(ids)
            graph.replay()
            return ids_out
        step.graph = graph
        return step

    def generate(self, prompt, steps, use_graph=True):
        """Greedy decoding: prompt (S, T) -> (S, steps) generated ids (int64)."""
        state = self.init_decode(prompt.shape[0], prompt.device)
        nxt = self.prefill(prompt, state)
        out = [nxt.clone()]
        step = self.decode_graph(state) if (use_graph and steps > 2) else (lambda ids: self.decode_step(ids, state))
        for _ in range(steps - 1):
            nxt = step(nxt)
            out.append(nxt.clone())
        return torch.stack(out, 1).long()


DEFAULTS = dict(d=256, layers=4, mlp_f=688, heads=4, n_sub=32, d_a=32, k=16)
ALLSDM_ARMS = ("onesdm_allsdm", "onesdm_allsdm_big")


def lm_kwargs(cfg):
    """cfg -> (merged cfg, the OneSdmLM keyword arguments it carries) (M:595-606)."""
    c = {**DEFAULTS, **cfg}
    mem_keys = ("heads", "n_sub", "d_a", "k", "learn_decay", "write_gate", "gate_bias", "read_mode", "out_norm",
                "addr_scale", "learn_scale", "chunk", "mem_in_grad", "out_norm_eps", "read_eps", "addr_bias", "tie", "seed",
                "reset_at_bos", "bos_id")
    arc_keys = ("arc_layers", "arc_d_c", "arc_n_sub", "arc_k", "arc_slot_keep", "arc_window", "arc_n_fetch", "arc_weighting")
    sdm_keys = ("sdm_heads", "sdm_d_a", "sdm_k", "sdm_scale", "sdm_learn_scale")
    kw = {kk: c[kk] for kk in mem_keys + arc_keys + sdm_keys if kk in c}
    if "decays" in c:
        kw["decays"] = tuple(c["decays"])
    return c, kw


def allsdm_n_sub(arm, c):
    """n_sub of the trained table (M:609-614)."""
    heads = c.get("sdm_heads", 4)
    d_a = c.get("sdm_d_a", 0) or min(32, (c["d"] // heads) // 2 * 2)
    n = c.get("sdm_n_sub", 0) or matched_sdm_n_sub(c["d"], c["mlp_f"], heads, d_a)
    return n * c.get("sdm_big_mult", 4) if arm == "onesdm_allsdm_big" else n


def build_onesdm(arm, V, cfg):
    """onesdm | plain | onesdm_allsdm | onesdm_allsdm_big (M:617-633).  The archive, sdmonly and transformer arms
    are comparison arms outside this path."""
    c, kw = lm_kwargs(cfg)
    if arm in ("onesdm", "plain"):
        return OneSdmLM(V, d=c["d"], layers=c["layers"], mlp_f=c["mlp_f"], mem=arm != "plain", archive=False, **kw)
    if arm in ALLSDM_ARMS:
        return OneSdmLM(V, d=c["d"], layers=c["layers"], mlp_f=c["mlp_f"], mem=True, archive=False, ffn="sdm",
                        sdm_n_sub=allsdm_n_sub(arm, c), **kw)
    raise ValueError(f"{arm}: not an arm of this path (onesdm, plain, onesdm_allsdm, onesdm_allsdm_big)")


def readme_fades(heads):
    """The trainer's default fades: 0, 0.8, 0.99, 1 repeated per 4 heads (track4_sdmonly_train.py:318-331)."""
    base = (0.0, 0.8, 0.99, 1.0)
    if heads % 4:
        raise ValueError("the default fades need a multiple of 4 heads")
    return base * (heads // 4)


def mlp_width(d):
    """8/3 d rounded up to a multiple of 16 (track4_sdmonly_train.py:334-336)."""
    return -(-d // 6) * 16


def decode_state_bytes(model, T=0):
    """Bytes kept to continue decoding (M:641-652): layers * h * M * (dh + 1) * 4, independent of T."""
    m = model.mems[0]
    return model.n_layers * m.h * m.M * (m.dh + 1) * 4 if model.has_mem else 0
