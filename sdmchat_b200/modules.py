"""Drop-in PyTorch modules for the SDMCHAT run-time SDM path, computed by libsdm_b200 (hand-written sm_100a CUDA).

Each class mirrors the reference class of the same name (constructor signature, parameter and buffer names,
state_dict keys, construction RNG order, attributes the reference's tests read) so a reference checkpoint loads
unchanged and `torch.manual_seed(s); Module(...)` gives the reference's weights.  The forward passes call the C ABI
(include/sdm_b200.h); there is no CPU or PyTorch fallback, and tensors must be on a CUDA device.

Reference files (inside the SDMCHAT project):
  M = experiments/track4/sdmllm/track4_onesdm_models.py
  L = experiments/track4/sdmllm/track4_sdmllm_models.py

Precision modes.  All-float32 parameters with float32 inputs run the float32 path (CUDA-core GEMMs, exact float32
products).  bfloat16 matrices with bfloat16 activations run the tensor-core path: activations and matrices in
bfloat16, float32 accumulation, float32 memory state, rounding exactly where a bfloat16 reference module rounds.
Small parameters (sub-keys, address bias, scales, fades, out-norm weights, gate bias) stay float32 in both.

Forward only: the backward pass is not built; calling a module with autograd recording raises.
"""
import math

import torch
import torch.nn as nn

from . import _lib as L_
from ._lib import check, lib, ptr, stream_ptr, workspace, dtype_code


def _forward_only(*tensors):
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors):
        raise NotImplementedError("libsdm_b200 builds the forward pass only: call the module under torch.no_grad()")


def _f32(t):
    return t.detach().to(torch.float32).contiguous()


def _cdt(t, dt):
    return t.detach().to(dt).contiguous()


def pk_address(z, keys1, keys2, k):
    """pk_address (M:134-148) on the GPU: z (N, h, d_a), keys (h, n_sub, d_a/2) -> scores (N, h, kk) descending,
    slot ids (N, h, kk) int64 in [0, n_sub^2).  Exactly equal scores are ordered lowest index first."""
    N, h, d_a = z.shape
    n_sub = keys1.shape[1]
    c1 = min(k, n_sub)
    kk = min(k, c1 * c1)
    zf, k1, k2 = _f32(z), _f32(keys1), _f32(keys2)
    sv = torch.empty(N, h, kk, dtype=torch.float32, device=z.device)
    si = torch.empty(N, h, kk, dtype=torch.int32, device=z.device)
    check(lib().sdm_pk_address(ptr(zf), ptr(k1), ptr(k2), N, h, d_a, n_sub, k, ptr(sv), ptr(si),
                               stream_ptr(z.device)), "sdm_pk_address")
    return sv, si.long()


class RMSNorm(nn.Module):
    """RMSNorm (L:63-71)."""

    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.w = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        _forward_only(x, self.w)
        x = x.contiguous()
        y = torch.empty_like(x)
        check(lib().sdm_rmsnorm(ptr(x), ptr(_cdt(self.w, x.dtype)), x.numel() // x.shape[-1], x.shape[-1], self.eps,
                                dtype_code(x.dtype), ptr(y), stream_ptr(x.device)), "sdm_rmsnorm")
        return y


class SwiGLU(nn.Module):
    """SwiGLU (L:89-97): forward(x) = down(silu(gate x) * up x); `block(x, norm_w)` computes x + SwiGLU(RMSNorm(x))
    in one call (M:544-545).  In bf16 the gate and up maps are one tensor-core GEMM against a packed weight (cached
    until a weight changes) whose epilogue forms silu(g) * u, so only the product reaches memory."""

    def __init__(self, d, f):
        super().__init__()
        self.gate = nn.Linear(d, f, bias=False)
        self.up = nn.Linear(d, f, bias=False)
        self.down = nn.Linear(f, d, bias=False)
        self._pcache = None

    def _packed(self, dt, device):
        """(packed gate|up weight (2f, d), down weight) in dtype dt, rebuilt only when a weight changes."""
        mats = (self.gate.weight, self.up.weight, self.down.weight)
        key = (dt, device) + tuple((t.data_ptr(), t._version) for t in mats)
        if self._pcache is not None and self._pcache[0] == key:
            return self._pcache[1]
        d, f = self.gate.in_features, self.gate.out_features
        wg, wu = _cdt(self.gate.weight, dt), _cdt(self.up.weight, dt)
        wgu = torch.empty(2 * f, d, dtype=dt, device=device)
        check(lib().sdm_swiglu_pack(ptr(wg), ptr(wu), d, f, dtype_code(dt), ptr(wgu), stream_ptr(device)),
              "sdm_swiglu_pack")
        keep = (wgu, _cdt(self.down.weight, dt))
        self._pcache = (key, keep)
        return keep

    def _run(self, x, norm_w, eps, add_residual, out=None):
        _forward_only(x, self.gate.weight)
        x = x.contiguous()
        d, f = self.gate.in_features, self.gate.out_features
        N = x.numel() // d
        dt = x.dtype
        wgu, wd = self._packed(dt, x.device)
        out = torch.empty_like(x) if out is None else out
        nw = None if norm_w is None else _cdt(norm_w, dt)
        ws = workspace(lib().sdm_swiglu_forward_workspace_size(N, d, f, dtype_code(dt)), x.device)
        check(lib().sdm_swiglu_forward(ptr(x), ptr(nw), ptr(wgu), ptr(wd), N, d, f, eps, dtype_code(dt),
                                       int(add_residual), ptr(out), ptr(ws), ws.numel(), stream_ptr(x.device)),
              "sdm_swiglu_forward")
        return out

    def forward(self, x):
        """SwiGLU.forward (L:96-97), in x's dtype."""
        return self._run(x, None, 0.0, False)

    def block(self, x, norm_w, eps=1e-6, out=None):
        """x + SwiGLU(RMSNorm(x)) with RMSNorm weight norm_w (OneSdmLM.residual, M:544-545)."""
        return self._run(x, norm_w, eps, True, out)


class RunTimeSdm(nn.Module):
    """A Kanerva memory with M = n_sub^2 hard locations per head, written and read while the text is read
    (M:151-300).  Same constructor, parameters, buffers and attributes as the reference."""

    def __init__(self, d, heads=4, n_sub=32, d_a=32, k=16, decays=(0.0, 0.8, 0.99, 1.0), learn_decay=False,
                 write_gate=True, gate_bias=0.0, read_mode="mean", out_norm=True, addr_scale=8.0, learn_scale=True,
                 chunk=128, read_eps=1e-3, mem_in_grad=1.0, out_norm_eps=1e-2, addr_bias=0.0, seed=0):
        super().__init__()
        assert d % heads == 0 and d_a % 2 == 0 and len(decays) == heads and read_mode in ("mean", "sum")
        g = torch.Generator().manual_seed(4321 + seed)
        self.d, self.h, self.dh, self.k, self.d_a, self.n_sub, self.M = d, heads, d // heads, k, d_a, n_sub, n_sub * n_sub
        self.chunk, self.read_mode, self.read_eps, self.mem_in_grad = chunk, read_mode, read_eps, mem_in_grad
        self.write_gate, self.out_norm, self.learn_decay = write_gate, out_norm, learn_decay
        self.out_norm_eps = out_norm_eps
        self.enabled = True
        self._leak = False
        self.norm = RMSNorm(d)
        self.wk = nn.Linear(d, heads * d_a, bias=False)
        self.wq = nn.Linear(d, heads * d_a, bias=False)
        self.wv = nn.Linear(d, d, bias=False)
        self.wg = nn.Linear(d, heads, bias=True)
        self.wo = nn.Linear(d, d, bias=False)
        self.keys1 = nn.Parameter(torch.randn(heads, n_sub, d_a // 2, generator=g))
        self.keys2 = nn.Parameter(torch.randn(heads, n_sub, d_a // 2, generator=g))
        self.addr_b = nn.Parameter(torch.randn(heads, d_a, generator=g) * addr_bias)
        self.log_scale = nn.Parameter(torch.full((heads,), math.log(addr_scale)), requires_grad=learn_scale)
        lam = torch.tensor(decays, dtype=torch.float32)
        if learn_decay:
            self.decay_logit = nn.Parameter(torch.logit(lam.clamp(1e-4, 1 - 1e-4)))
        else:
            self.register_buffer("decays_fixed", lam, persistent=True)
        if out_norm:
            self.onorm_w = nn.Parameter(torch.ones(heads, self.dh))
        self.gate_bias0 = gate_bias
        self._pcache = None

    def reset_init(self):
        nn.init.zeros_(self.wo.weight)
        nn.init.zeros_(self.wg.weight)
        nn.init.constant_(self.wg.bias, self.gate_bias0)

    def decay(self):
        return torch.sigmoid(self.decay_logit) if self.learn_decay else self.decays_fixed

    # -------------------------------------------------------------------------------------- C ABI parameters
    def _params(self, dt):
        """sdm_rt_params for compute dtype dt, with the stacked projection [wk; wq; wv; wg] cached until any
        parameter changes (keyed on tensor versions)."""
        mats = (self.norm.w, self.wk.weight, self.wq.weight, self.wv.weight, self.wg.weight, self.wg.bias,
                self.wo.weight, self.keys1, self.keys2, self.addr_b, self.log_scale,
                self.decay_logit if self.learn_decay else self.decays_fixed,
                self.onorm_w if self.out_norm else self.log_scale)
        key = (dt, self.write_gate, self.read_mode, self.out_norm) + tuple((t.data_ptr(), t._version) for t in mats)
        if self._pcache is not None and self._pcache[0] == key:
            return self._pcache[1]
        keep = {
            "norm_w": _cdt(self.norm.w, dt),
            "w_proj": torch.cat([self.wk.weight, self.wq.weight, self.wv.weight, self.wg.weight], 0).detach().to(dt).contiguous(),
            "wg_bias": _f32(self.wg.bias), "wo": _cdt(self.wo.weight, dt),
            "keys1": _f32(self.keys1), "keys2": _f32(self.keys2), "addr_b": _f32(self.addr_b),
            "log_scale": _f32(self.log_scale), "decay": _f32(self.decay()),
            "onorm_w": _f32(self.onorm_w) if self.out_norm else None,
        }
        p = L_.RtParams(d=self.d, heads=self.h, n_sub=self.n_sub, d_a=self.d_a, k=self.k,
                        write_gate=int(bool(self.write_gate)), read_sum=int(self.read_mode == "sum"),
                        out_norm=int(bool(self.out_norm)), read_eps=self.read_eps, out_norm_eps=self.out_norm_eps,
                        norm_eps=self.norm.eps, dtype=dtype_code(dt),
                        **{k: (v.data_ptr() if v is not None else None) for k, v in keep.items()})
        self._pcache = (key, (p, keep))
        return p, keep

    def _sel_k(self):
        c1 = min(self.k, self.n_sub)
        return min(self.k, c1 * c1)

    def _run(self, x, reset=None, add_residual=False, want=()):
        """One sdm_rt_forward call.  want: names of the optional outputs to return."""
        _forward_only(x, self.wk.weight)
        if self._leak:
            raise NotImplementedError("the reference's causality-leak control (_leak) is a test-only switch of the "
                                      "PyTorch module and is not built into the kernels")
        x = x.contiguous()
        B, T, _ = x.shape
        dt = x.dtype
        p, _ = self._params(dt)
        dev = x.device
        kk, h = self._sel_k(), self.h
        f32 = dict(dtype=torch.float32, device=dev)
        out = torch.empty_like(x)
        mem = torch.empty(B, h, self.M, self.dh, **f32)
        cnt = torch.empty(B, h, self.M, **f32)
        gate = torch.empty(B, T, h, **f32)
        o = {}
        if "sel" in want:
            o["siw"] = torch.empty(B, h, T, kk, dtype=torch.int32, device=dev)
            o["sir"] = torch.empty(B, h, T, kk, dtype=torch.int32, device=dev)
            o["ww"] = torch.empty(B, h, T, kk, **f32)
            o["wr"] = torch.empty(B, h, T, kk, **f32)
        if "values" in want:
            o["V"] = torch.empty(B, T, self.d, **f32)
        if "z" in want:
            o["z"] = torch.empty(B, T, 2, h, self.d_a, **f32)
        if "read" in want:
            o["num"] = torch.empty(B, T, h, self.dh, **f32)
            o["den"] = torch.empty(B, T, h, **f32)
        rs = None
        if reset is not None:
            rs = reset.to(device=dev, dtype=torch.uint8).contiguous()
        ws = workspace(lib().sdm_rt_forward_workspace_size(p, B, T), dev)
        check(lib().sdm_rt_forward(p, ptr(x), B, T, ptr(rs), int(add_residual), ptr(out), ptr(mem), ptr(cnt),
                                   ptr(o.get("siw")), ptr(o.get("ww")), ptr(o.get("sir")), ptr(o.get("wr")),
                                   ptr(gate), ptr(o.get("V")), ptr(o.get("z")), ptr(o.get("num")), ptr(o.get("den")),
                                   ptr(ws), ws.numel(), stream_ptr(dev)), "sdm_rt_forward")
        self.last_state = (mem, cnt)
        self.last_gate = gate
        return out, o

    def prepare(self, x):
        """RunTimeSdm.prepare (M:195-213): siw, ww, sir, wr (B, h, T, k) and V (B, h, T, dh)."""
        B, T, _ = x.shape
        _, o = self._run(x, want=("sel", "values"))
        V = o["V"].view(B, T, self.h, self.dh).transpose(1, 2)
        return o["siw"].long(), o["ww"], o["sir"].long(), o["wr"], V

    def _chunk(self, siw, ww, sir, wr, Vc, mem, cnt, lam, seg=None, seg_prev=None):
        """RunTimeSdm._chunk (M:215-241): one chunk of the write-then-read from the carried state (mem (B,h,M,dh),
        cnt (B,h,M)).  siw, sir (B,h,L,k); ww, wr (B,h,L,k); Vc (B,h,L,dh); lam (h,); seg (B,L) / seg_prev (B,):
        segment numbers (a change empties the memory before that position reads).  Returns num (B,h,L,dh),
        den (B,h,L,1) and the state after the chunk, all float32."""
        _forward_only(Vc, ww, wr, mem)
        if self._leak:
            raise NotImplementedError("the reference's causality-leak control (_leak) is a test-only switch of the "
                                      "PyTorch module and is not built into the kernels")
        B, h, L, k = siw.shape
        dev = Vc.device
        f32 = dict(dtype=torch.float32, device=dev)
        i32 = lambda t: t.detach().to(device=dev, dtype=torch.int32).contiguous()  # noqa: E731
        sel = [i32(siw), _f32(ww), i32(sir), _f32(wr)]
        V = Vc.detach().float().transpose(1, 2).reshape(B * L, h * self.dh).contiguous()  # token-major rows
        rs = None
        if seg is not None:
            prev = torch.cat([seg_prev.reshape(B, 1).to(seg.dtype), seg[:, :-1]], 1)
            rs = (seg != prev).to(torch.uint8).contiguous()
        mem_in, cnt_in = _f32(mem), _f32(cnt)
        lam_d = _f32(lam).to(dev)
        num = torch.empty(B, L, h, self.dh, **f32)
        den = torch.empty(B, L, h, **f32)
        mem_o = torch.empty(B, h, self.M, self.dh, **f32)
        cnt_o = torch.empty(B, h, self.M, **f32)
        ws = workspace(lib().sdm_rt_scan_workspace_size(B, L, h, k), dev)
        check(lib().sdm_rt_scan(*(ptr(t) for t in sel), ptr(V), h * self.dh, ptr(lam_d), ptr(rs), B, L, h, self.n_sub,
                                self.dh, k, ptr(mem_in), ptr(cnt_in), ptr(num), ptr(den), ptr(mem_o), ptr(cnt_o),
                                ptr(ws), ws.numel(), stream_ptr(dev)), "sdm_rt_scan")
        return num.transpose(1, 2), den.transpose(1, 2)[..., None], mem_o, cnt_o

    def finish(self, num, den, B, T, dtype):
        """RunTimeSdm.finish (M:243-247): num (B,h,T,dh), den (B,h,T,1) -> wo(out-normed read) (B,T,d) in dtype."""
        _forward_only(num, den, self.wo.weight)
        dev = num.device
        p, _ = self._params(dtype)
        n = num.detach().float().transpose(1, 2).contiguous()          # (B, T, h, dh)
        dn = den.detach().float().reshape(B, self.h, T).transpose(1, 2).contiguous()  # (B, T, h)
        out = torch.empty(B, T, self.d, dtype=dtype, device=dev)
        ws = workspace(lib().sdm_rt_finish_workspace_size(p, B * T), dev)
        check(lib().sdm_rt_finish(p, ptr(n), ptr(dn), B * T, None, ptr(out), ptr(ws), ws.numel(), stream_ptr(dev)),
              "sdm_rt_finish")
        return out

    def forward(self, x, reset=None):
        """RunTimeSdm.forward (M:249-274): every call starts from an empty memory; reset (B, T) bool empties it
        before that position reads.  Sets last_state = (mem (B,h,M,dh), cnt (B,h,M)) and last_gate."""
        if not self.enabled:
            return torch.zeros_like(x)
        return self._run(x, reset)[0]

    def forward_with(self, x, reset=None, add_residual=False, want=("sel", "values", "read")):
        """forward plus the intermediates the kernels produce (selections, values, num/den)."""
        return self._run(x, reset, add_residual, want)

    # ---------------------------------------------------------------------------------------------- decode
    def init_state(self, S, device):
        """An empty carried state for S streams: mem (S,h,M,dh), cnt (S,h,M), scale (S,h), last_w (S,h,k)."""
        f32 = dict(dtype=torch.float32, device=device)
        return {"mem": torch.zeros(S, self.h, self.M, self.dh, **f32), "cnt": torch.zeros(S, self.h, self.M, **f32),
                "scale": torch.ones(S, self.h, **f32),
                "last_w": torch.full((S, self.h, self._sel_k()), -1, dtype=torch.int32, device=device)}

    def decode_step(self, x, state, reset=None, add_residual=False, out=None):
        """One token per stream (x (S, d)) through the memory, reading then writing the carried state in place."""
        _forward_only(x, self.wk.weight)
        x = x.contiguous()
        S = x.shape[0]
        p, _ = self._params(x.dtype)
        out = torch.empty_like(x) if out is None else out
        rs = None if reset is None else reset.to(device=x.device, dtype=torch.uint8).contiguous()
        ws = workspace(lib().sdm_rt_decode_workspace_size(p, S), x.device)
        check(lib().sdm_rt_decode_step(p, ptr(x), S, ptr(rs), int(add_residual), ptr(out), ptr(state["mem"]),
                                       ptr(state["cnt"]), ptr(state["scale"]), ptr(state["last_w"]), ptr(ws),
                                       ws.numel(), stream_ptr(x.device)), "sdm_rt_decode_step")
        return out

    def forward_sequential(self, x, reset=None):
        """RunTimeSdm.forward_sequential (M:276-300): the token recurrence, here T carried-state decode steps
        from an empty memory.  Sets last_state to the true (mem, cnt)."""
        if not self.enabled:
            return torch.zeros_like(x)
        B, T, _ = x.shape
        st = self.init_state(B, x.device)
        outs = []
        for t in range(T):
            outs.append(self.decode_step(x[:, t], st, None if reset is None else reset[:, t]))
        sc = st["scale"]
        self.last_state = (st["mem"] * sc[..., None, None], st["cnt"] * sc[..., None])
        return torch.stack(outs, 1)


class TrainedSdm(nn.Module):
    """The trained product-key table of the FULL arm (M:414-457), same constructor and parameters."""

    def __init__(self, d, n_sub, heads=4, d_a=32, k=32, scale=8.0, learn_scale=True, seed=0):
        super().__init__()
        assert d % heads == 0 and d_a % 2 == 0 and heads * d_a <= d
        g = torch.Generator().manual_seed(9876 + seed)
        self.d, self.h, self.dh, self.d_a, self.k = d, heads, d // heads, d_a, k
        self.n_sub, self.M = n_sub, n_sub * n_sub
        self.norm = RMSNorm(d)
        self.wq = nn.Linear(d, heads * d_a, bias=False)
        self.keys1 = nn.Parameter(torch.randn(heads, n_sub, d_a // 2, generator=g))
        self.keys2 = nn.Parameter(torch.randn(heads, n_sub, d_a // 2, generator=g))
        self.values = nn.Parameter(torch.zeros(heads, self.M, self.dh))
        self.log_scale = nn.Parameter(torch.full((heads,), math.log(scale)), requires_grad=learn_scale)
        self.wo = nn.Linear(d, d, bias=False)
        self._pcache = None

    def reset_init(self):
        nn.init.zeros_(self.values)

    def _params(self, dt):
        mats = (self.norm.w, self.wq.weight, self.keys1, self.keys2, self.values, self.log_scale, self.wo.weight)
        key = (dt,) + tuple((t.data_ptr(), t._version) for t in mats)
        if self._pcache is not None and self._pcache[0] == key:
            return self._pcache[1]
        keep = {"norm_w": _cdt(self.norm.w, dt), "wq": _cdt(self.wq.weight, dt), "keys1": _f32(self.keys1),
                "keys2": _f32(self.keys2), "values": _cdt(self.values, dt), "log_scale": _f32(self.log_scale),
                "wo": _cdt(self.wo.weight, dt)}
        p = L_.TsParams(d=self.d, heads=self.h, n_sub=self.n_sub, d_a=self.d_a, k=self.k, norm_eps=self.norm.eps,
                        dtype=dtype_code(dt), **{k: v.data_ptr() for k, v in keep.items()})
        self._pcache = (key, (p, keep))
        return p, keep

    def _run(self, x, add_residual=False, want_sel=False, out=None, want_q=False):
        """One sdm_ts_forward call: (out, slot ids, weights[, queries (N, h, d_a) when want_q])."""
        _forward_only(x, self.wq.weight)
        x = x.contiguous()
        N = x.numel() // self.d
        p, _ = self._params(x.dtype)
        c1 = min(self.k, self.n_sub)
        kk = min(self.k, c1 * c1)
        out = torch.empty_like(x) if out is None else out
        si = w = q = None
        if want_sel:
            si = torch.empty(N, self.h, kk, dtype=torch.int32, device=x.device)
            w = torch.empty(N, self.h, kk, dtype=torch.float32, device=x.device)
        if want_q:
            q = torch.empty(N, self.h, self.d_a, dtype=torch.float32, device=x.device)
        ws = workspace(lib().sdm_ts_forward_workspace_size(p, N), x.device)
        check(lib().sdm_ts_forward(p, ptr(x), N, int(add_residual), ptr(out), ptr(si), ptr(w), ptr(q), ptr(ws),
                                   ws.numel(), stream_ptr(x.device)), "sdm_ts_forward")
        return (out, si, w, q) if want_q else (out, si, w)

    def address(self, x):
        """TrainedSdm.address (M:438-446): soft weights (N, h, k) and slot ids (N, h, k)."""
        _, si, w = self._run(x, want_sel=True)
        return w, si.long()

    def forward(self, x):
        out, si, _ = self._run(x, want_sel=True)
        self.last_si = si.long()
        return out


def trained_sdm_params(d, n_sub, heads, d_a):
    """Parameter count of one TrainedSdm (M:460-462)."""
    return d + d * heads * d_a + heads * n_sub * d_a + heads * n_sub * n_sub * (d // heads) + heads + d * d


def matched_sdm_n_sub(d, mlp_f, heads, d_a):
    """The n_sub whose TrainedSdm weight count is closest to one SwiGLU(d, mlp_f) plus its RMSNorm (M:465-468)."""
    target = 3 * d * mlp_f + d
    return min(range(2, 4097), key=lambda n: abs(trained_sdm_params(d, n, heads, d_a) - target))
