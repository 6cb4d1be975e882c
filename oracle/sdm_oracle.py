"""CPU oracle for the SDMCHAT run-time SDM path: a numpy float32 restatement of the reference algorithm.

TEST INFRASTRUCTURE ONLY. Nothing in the product (the ``sdmchat_b200`` package or its CUDA library) imports, calls
or links this file; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg use it, and
there only as the checker or the timed CPU baseline.

Reference files (paths inside the TripleSparkleAI/SDMCHAT project):
  M = experiments/track4/sdmllm/track4_onesdm_models.py
  L = experiments/track4/sdmllm/track4_sdmllm_models.py

Parity is pinned: ``tests/test_oracle_golden.py`` checks every function here against golden vectors produced by
the reference module itself (``tests/golden/make_golden.py`` imports the unmodified reference and writes them).

Numerics.  Every array is float32 and every step rounds as the reference's CPU float32 path does.  A "bf16 stream"
mode reproduces the reference run with a bfloat16 residual stream (the reference's RMSNorm casts its result back to
the input dtype, L:69-71): the normalised activations are rounded to bfloat16, the bfloat16 matmuls round their
outputs, and the residual adds round.  Top-k ties are broken lowest-index-first here; the reference's order among
exactly equal scores is whatever ``aten::topk`` does and is outside the parity contract, so tests compare selections
only where the k-th / (k+1)-th score margin is non-zero (and report near-ties with their margins).
"""
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

F32 = np.float32

# Row-independent steps (product-key addressing, bfloat16 rounding of large arrays) run on row blocks in threads;
# numpy releases the GIL inside these kernels, so the blocks use the host's cores.  Results do not depend on the
# split.  SDM_ORACLE_THREADS=1 runs everything on the calling thread.
_THREADS = int(os.environ.get("SDM_ORACLE_THREADS", "0")) or (os.cpu_count() or 1)
_POOL = None


def _pool():
    global _POOL
    if _POOL is None:
        _POOL = ThreadPoolExecutor(max_workers=_THREADS)
    return _POOL


def _row_blocks(n, min_rows):
    """[(lo, hi)] row ranges for the thread pool (one range when the work is small or threads are off)."""
    nb = min(_THREADS, max(1, n // min_rows))
    if nb <= 1:
        return [(0, n)]
    step = -(-n // nb)
    return [(lo, min(n, lo + step)) for lo in range(0, n, step)]


# ----------------------------------------------------------------------------------------------- numeric helpers
def bf16(a):
    """Round float32 values to the nearest bfloat16 (ties to even), returned as float32 (torch's conversion)."""
    a = np.ascontiguousarray(a, dtype=F32)
    if a.size >= (1 << 22) and a.ndim >= 1:
        flat = a.reshape(a.shape[0], -1) if a.ndim > 1 else a.reshape(-1, 1)
        out = np.empty_like(flat)
        blocks = _row_blocks(flat.shape[0], 1)

        def run(lohi):
            lo, hi = lohi
            out[lo:hi] = _bf16_block(flat[lo:hi])

        list(_pool().map(run, blocks))
        return out.reshape(a.shape)
    return _bf16_block(a)


def _bf16_block(a):
    u = a.view(np.uint32)
    r = (u >> 16) & np.uint32(1)
    r += np.uint32(0x7FFF)
    r += u  # finite values only: the carry of the largest ones rounds them to infinity, as the conversion does
    r &= np.uint32(0xFFFF0000)
    return r.view(F32).reshape(a.shape)


def _order_keys(s):
    """uint64 keys whose ascending order is the (score descending, index ascending) order of s along the last axis;
    -0.0 and +0.0 get the same score part (they compare equal)."""
    v = np.ascontiguousarray(s, dtype=F32) + F32(0)
    m = v.view(np.int32) >> 31  # -1 for negative values, 0 otherwise
    m |= np.int32(-0x80000000)
    desc = ~(v.view(np.int32) ^ m)  # as uint32: ascending = the float value descending
    key = desc.view(np.uint32).astype(np.uint64)
    key <<= np.uint64(32)
    key |= np.arange(s.shape[-1], dtype=np.uint64)
    return key


def topk_desc(s, c):
    """Top-c along the last axis, descending, ties lowest-index-first. Returns (values, indices int64)."""
    n = s.shape[-1]
    key = _order_keys(s)
    if c < n:
        key = np.partition(key, c - 1, axis=-1)[..., :c]  # keys are distinct: the selected set is exact
    key = np.sort(key, axis=-1)
    idx = (key & np.uint64(0xFFFFFFFF)).astype(np.int64)
    return np.take_along_axis(s, idx, -1), idx


def softmax(x):
    m = x.max(-1, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(-1, keepdims=True)).astype(F32, copy=False)


def sigmoid(x):
    return (F32(1) / (F32(1) + np.exp(-x))).astype(F32, copy=False)


def silu(x):
    return (x / (F32(1) + np.exp(-x))).astype(F32, copy=False)


def l2_normalize(v):
    """F.normalize(v, dim=-1): v / max(||v||_2, 1e-12)."""
    n = np.sqrt((v * v).sum(-1, keepdims=True))
    return (v / np.maximum(n, F32(1e-12))).astype(F32, copy=False)


def rmsnorm(x, w, eps=1e-6, bf16_stream=False):
    """RMSNorm.forward (L:69-71): (x * rsqrt(mean x^2 + eps)).to(x.dtype) * w; with a bf16 stream both the cast
    and the product with the bf16 weight round to bfloat16."""
    x = x.astype(F32, copy=False)
    r = F32(1) / np.sqrt((x * x).mean(-1, keepdims=True, dtype=F32) + F32(eps))
    y = (x * r).astype(F32, copy=False)
    if bf16_stream:
        return bf16(bf16(y) * w)
    return (y * w).astype(F32, copy=False)


def linear(x, w, bf16_out=False):
    """nn.Linear without bias: x @ w.T in float32 (a bf16 matmul accumulates in float32, then rounds)."""
    y = np.matmul(x.astype(F32, copy=False), w.astype(F32, copy=False).T).astype(F32, copy=False)
    return bf16(y) if bf16_out else y


# ------------------------------------------------------------------------------------------- product-key address
def pk_address(z, keys1, keys2, k, return_margin=False, force_si=None):
    """pk_address (M:134-148) over row blocks of z in threads; see _pk_address_rows."""
    blocks = _row_blocks(z.shape[0], 1024)
    if len(blocks) == 1:
        return _pk_address_rows(z, keys1, keys2, k, return_margin, force_si)
    parts = list(_pool().map(lambda lh: _pk_address_rows(
        z[lh[0]:lh[1]], keys1, keys2, k, return_margin,
        None if force_si is None else np.asarray(force_si)[lh[0]:lh[1]]), blocks))
    return tuple(np.concatenate([p[i] for p in parts], 0) for i in range(len(parts[0])))


def _pk_address_rows(z, keys1, keys2, k, return_margin=False, force_si=None):
    """pk_address (M:134-148). z (N, h, d_a), keys (h, n_sub, d_a/2) -> scores (N, h, kk) descending and slot ids
    (N, h, kk) in [0, n_sub^2).  With return_margin, also the brute-force gap between the kk-th and (kk+1)-th score
    of the full n_sub x n_sub grid (inf when kk = n_sub^2): a selection is only defined where that gap is > 0.
    force_si (N, h, kk) (a checker's teacher forcing): return these slot ids, in the given order, with their scores
    (s1[a] + s2[b]) / 2, instead of this function's own selection (margins still describe its own)."""
    z = z.astype(F32, copy=False)
    half = z.shape[-1] // 2
    n_sub = keys1.shape[1]
    z1, z2 = l2_normalize(z[..., :half]), l2_normalize(z[..., half:])
    k1, k2 = l2_normalize(keys1.astype(F32, copy=False)), l2_normalize(keys2.astype(F32, copy=False))
    s1 = np.einsum("nhd,hsd->nhs", z1, k1).astype(F32, copy=False)
    s2 = np.einsum("nhd,hsd->nhs", z2, k2).astype(F32, copy=False)
    c1 = min(k, n_sub)
    v1, i1 = topk_desc(s1, c1)
    v2, i2 = topk_desc(s2, c1)
    comb = ((v1[..., :, None] + v2[..., None, :]) * F32(0.5)).astype(F32, copy=False)
    comb = comb.reshape(comb.shape[:-2] + (c1 * c1,))
    kk = min(k, c1 * c1)
    sv, sc = topk_desc(comb, kk)
    a = sc // c1
    si = np.take_along_axis(i1, a, -1) * n_sub + np.take_along_axis(i2, sc - a * c1, -1)
    if force_si is not None:
        si = np.asarray(force_si).astype(np.int64).reshape(si.shape)
        sv = ((np.take_along_axis(s1, si // n_sub, -1) + np.take_along_axis(s2, si % n_sub, -1))
              * F32(0.5)).astype(F32, copy=False)
    if not return_margin:
        return sv, si
    full = ((s1[..., :, None] + s2[..., None, :]) * F32(0.5)).astype(F32, copy=False).reshape(s1.shape[:-1] + (n_sub * n_sub,))
    if kk >= n_sub * n_sub:
        margin = np.full(full.shape[:-1], np.inf, F32)
    else:
        part = -np.sort(-full, axis=-1)
        margin = (part[..., kk - 1] - part[..., kk]).astype(F32, copy=False)
    return sv, si, margin


# -------------------------------------------------------------------------------------------------- RunTimeSdm
class RunTimeSdmParams:
    """The parameters of one RunTimeSdm (M:154-185), as float32 numpy arrays.  ``from_state_dict`` accepts the
    reference's state_dict keys (norm.w, wk.weight, wq.weight, wv.weight, wg.weight, wg.bias, wo.weight, keys1,
    keys2, addr_b, log_scale, decays_fixed | decay_logit, onorm_w)."""

    def __init__(self, sd, heads, n_sub, d_a, k, write_gate=True, read_mode="mean", out_norm=True, read_eps=1e-3,
                 out_norm_eps=1e-2):
        g = {kk: np.asarray(v, dtype=F32) for kk, v in sd.items()}
        self.norm_w, self.wk, self.wq, self.wv = g["norm.w"], g["wk.weight"], g["wq.weight"], g["wv.weight"]
        self.wg, self.bg, self.wo = g["wg.weight"], g["wg.bias"], g["wo.weight"]
        self.keys1, self.keys2, self.addr_b, self.log_scale = g["keys1"], g["keys2"], g["addr_b"], g["log_scale"]
        if "decays_fixed" in g:
            self.lam = g["decays_fixed"]
        else:
            self.lam = sigmoid(g["decay_logit"])  # RunTimeSdm.decay (M:192-193)
        self.onorm_w = g.get("onorm_w")
        self.d = self.wv.shape[0]
        self.h, self.n_sub, self.d_a, self.k = heads, n_sub, d_a, k
        self.dh, self.M = self.d // heads, n_sub * n_sub
        self.write_gate, self.read_mode, self.out_norm = write_gate, read_mode, out_norm
        self.read_eps, self.out_norm_eps = F32(read_eps), F32(out_norm_eps)


def rt_prepare(p, x, bf16_stream=False, margins=True, force=None):
    """RunTimeSdm.prepare (M:195-213): x (B, T, d) -> siw, ww, sir, wr (B, h, T, k), V (B, h, T, dh), gate
    (B, T, h), and (with margins) the address margins of the write and read selections (B, h, T).  force: a dict
    with the slot ids siw, sir (B, h, T, k) to use instead of this function's own (teacher forcing)."""
    B, T, _ = x.shape
    hx = rmsnorm(x, p.norm_w, bf16_stream=bf16_stream).reshape(B * T, p.d)
    kz = linear(hx, p.wk).reshape(B * T, p.h, p.d_a) + p.addr_b
    qz = linear(hx, p.wq).reshape(B * T, p.h, p.d_a) + p.addr_b

    def tok(t):  # (B, h, T, k) -> (B*T, h, k)
        return None if t is None else np.asarray(t).transpose(0, 2, 1, 3).reshape(B * T, p.h, -1)
    fw, fr = (tok(force.get("siw")), tok(force.get("sir"))) if force else (None, None)
    if margins:
        svw, siw, mw = pk_address(kz, p.keys1, p.keys2, p.k, return_margin=True, force_si=fw)
        svr, sir, mr = pk_address(qz, p.keys1, p.keys2, p.k, return_margin=True, force_si=fr)
    else:
        (svw, siw), (svr, sir) = (pk_address(kz, p.keys1, p.keys2, p.k, force_si=fw),
                                  pk_address(qz, p.keys1, p.keys2, p.k, force_si=fr))
        mw = mr = np.full(siw.shape[:2], np.inf, F32)
    scale = np.exp(p.log_scale)[None, :, None].astype(F32, copy=False)
    ww = softmax((svw * scale).astype(F32, copy=False))
    wr = softmax((svr * scale).astype(F32, copy=False))
    if p.write_gate:
        gate = sigmoid((linear(hx, p.wg) + p.bg).astype(F32, copy=False))
    else:
        gate = np.ones((B * T, p.h), F32)
    ww = (ww * gate.reshape(B * T, p.h, 1)).astype(F32, copy=False)
    c = siw.shape[-1]

    def bh(t):
        return np.ascontiguousarray(t.reshape(B, T, p.h, c).transpose(0, 2, 1, 3))
    V = np.ascontiguousarray(linear(hx, p.wv).reshape(B, T, p.h, p.dh).transpose(0, 2, 1, 3))
    return dict(siw=bh(siw), ww=bh(ww), sir=bh(sir), wr=bh(wr), V=V, gate=gate.reshape(B, T, p.h),
                kz=kz, qz=qz, margin_w=mw.reshape(B, T, p.h).transpose(0, 2, 1),
                margin_r=mr.reshape(B, T, p.h).transpose(0, 2, 1))


def rt_chunk(siw, ww, sir, wr, Vc, mem, cnt, lam, M, seg=None, seg_prev=None):
    """RunTimeSdm._chunk (M:215-241): one chunk of the parallel write-then-read with the carried state."""
    B, h, L, _ = siw.shape
    A = np.zeros((B, h, L, M), F32)
    Rq = np.zeros((B, h, L, M), F32)
    bi, hi, li = np.meshgrid(np.arange(B), np.arange(h), np.arange(L), indexing="ij")
    for j in range(siw.shape[-1]):
        np.add.at(A, (bi, hi, li, siw[..., j]), ww[..., j])
        np.add.at(Rq, (bi, hi, li, sir[..., j]), wr[..., j])
    pos = np.arange(L, dtype=F32)
    e = pos[:, None] - 1 - pos[None, :]
    mask = (e >= 0).astype(F32, copy=False)
    lam_ = lam.astype(F32, copy=False)[None, :, None, None]
    D = np.power(lam_, np.maximum(e, 0)).astype(F32, copy=False) * mask
    fade_in = np.power(lam_, pos[None, None, :, None]).astype(F32, copy=False)
    tail = np.power(lam_, (L - 1 - pos)[None, None, :, None]).astype(F32, copy=False)
    keep = F32(1)
    if seg is not None:
        D = D * (seg[:, :, None] == seg[:, None, :]).astype(F32, copy=False)[:, None]
        fade_in = fade_in * (seg == seg_prev[:, None]).astype(F32, copy=False)[:, None, :, None]
        tail = tail * (seg == seg[:, -1:]).astype(F32, copy=False)[:, None, :, None]
        keep = (seg[:, -1] == seg_prev).astype(F32, copy=False)[:, None, None]
    ov = (np.matmul(Rq, A.transpose(0, 1, 3, 2)) * D).astype(F32, copy=False)
    num = (np.matmul(ov, Vc) + np.matmul(Rq, mem) * fade_in).astype(F32, copy=False)
    den = (ov.sum(-1, keepdims=True) + np.matmul(Rq, cnt[..., None]) * fade_in).astype(F32, copy=False)
    At = (A * tail).astype(F32, copy=False)
    keep_m = keep if seg is None else keep[..., None]
    mem = (mem * np.power(lam_, F32(L)) * keep_m + np.matmul(At.transpose(0, 1, 3, 2), Vc)).astype(F32, copy=False)
    cnt = (cnt * np.power(lam.astype(F32, copy=False)[None, :, None], F32(L)) * keep + At.sum(2)).astype(F32, copy=False)
    return num, den, mem, cnt


def rt_scan(prep, lam, M, chunk=128, reset=None):
    """The chunk loop of RunTimeSdm.forward (M:255-273): returns num (B, h, T, dh), den (B, h, T, 1), and the
    final state mem (B, h, M, dh), cnt (B, h, M).  reset (B, T) bool empties the memory before a position reads."""
    siw, ww, sir, wr, V = prep["siw"], prep["ww"], prep["sir"], prep["wr"], prep["V"]
    B, h, T, dh = V.shape
    mem = np.zeros((B, h, M, dh), F32)
    cnt = np.zeros((B, h, M), F32)
    seg = None if reset is None else np.cumsum(reset.astype(np.int64), 1)
    nums, dens = [], []
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        args = (siw[:, :, c0:c1], ww[:, :, c0:c1], sir[:, :, c0:c1], wr[:, :, c0:c1], V[:, :, c0:c1], mem, cnt, lam, M)
        kw = {}
        if seg is not None:
            kw = dict(seg=seg[:, c0:c1], seg_prev=seg[:, c0 - 1] if c0 > 0 else np.zeros_like(seg[:, 0]))
        n_, d_, mem, cnt = rt_chunk(*args, **kw)
        nums.append(n_)
        dens.append(d_)
    return np.concatenate(nums, 2), np.concatenate(dens, 2), mem, cnt


def rt_scan_sequential(prep, lam, M, reset=None, mem=None, cnt=None):
    """RunTimeSdm.forward_sequential's token loop (M:285-299): read k rows BEFORE the write, then decay the whole
    state and write k rows.  An initial (mem, cnt) may be given (carried-state decode: the state after a prefix)."""
    siw, ww, sir, wr, V = prep["siw"], prep["ww"], prep["sir"], prep["wr"], prep["V"]
    B, h, T, dh = V.shape
    mem = np.zeros((B, h, M, dh), F32) if mem is None else mem.astype(F32, copy=False).copy()
    cnt = np.zeros((B, h, M), F32) if cnt is None else cnt.astype(F32, copy=False).copy()
    lam3 = lam.astype(F32, copy=False)[None, :, None]
    nums, dens = [], []
    bi, hi = np.meshgrid(np.arange(B), np.arange(h), indexing="ij")
    for t in range(T):
        if reset is not None:
            live = (~reset[:, t]).astype(F32, copy=False)[:, None, None]
            mem, cnt = mem * live[..., None], cnt * live
        rows = sir[:, :, t]
        got = mem[bi[..., None], hi[..., None], rows]  # (B, h, k, dh)
        nums.append((wr[:, :, t, :, None] * got).sum(2).astype(F32, copy=False))
        dens.append((wr[:, :, t] * cnt[bi[..., None], hi[..., None], rows]).sum(-1, keepdims=True).astype(F32, copy=False))
        add = np.zeros_like(mem)
        addc = np.zeros_like(cnt)
        wrow = siw[:, :, t]
        for j in range(wrow.shape[-1]):
            np.add.at(add, (bi, hi, wrow[..., j]), ww[:, :, t, j, None] * V[:, :, t])
            np.add.at(addc, (bi, hi, wrow[..., j]), ww[:, :, t, j])
        mem = (mem * lam3[..., None] + add).astype(F32, copy=False)
        cnt = (cnt * lam3 + addc).astype(F32, copy=False)
    return np.stack(nums, 2), np.stack(dens, 2), mem, cnt


def rt_finish(p, num, den, bf16_out=False):
    """RunTimeSdm.finish (M:243-247): mean (or sum) read, per-head RMS out-norm, then wo; num (B, h, T, dh)."""
    B, h, T, dh = num.shape
    r = (num / (den + p.read_eps)).astype(F32, copy=False) if p.read_mode == "mean" else num
    if p.out_norm:
        rs = F32(1) / np.sqrt((r * r).mean(-1, keepdims=True, dtype=F32) + p.out_norm_eps)
        r = (r * rs).astype(F32, copy=False) * p.onorm_w[None, :, None, :]
    y = r.transpose(0, 2, 1, 3).reshape(B, T, p.d)
    return linear(y, p.wo, bf16_out=bf16_out)


def rt_forward(p, x, chunk=128, reset=None, bf16_stream=False, sequential=False, margins=True, force=None):
    """RunTimeSdm.forward (M:249-274) / forward_sequential (M:276-300): returns (out, dict of intermediates).
    force: slot ids to use instead of the oracle's own (see rt_prepare)."""
    prep = rt_prepare(p, x, bf16_stream, margins, force)
    if sequential:
        num, den, mem, cnt = rt_scan_sequential(prep, p.lam, p.M, reset)
    else:
        num, den, mem, cnt = rt_scan(prep, p.lam, p.M, chunk, reset)
    out = rt_finish(p, num, den, bf16_out=bf16_stream)
    prep.update(num=num, den=den, mem=mem, cnt=cnt)
    return out, prep


# -------------------------------------------------------------------------------------- TrainedSdm, SwiGLU, stack
class TrainedSdmParams:
    """TrainedSdm (M:414-457) parameters: norm.w, wq.weight, keys1, keys2, values, log_scale, wo.weight."""

    def __init__(self, sd, heads, n_sub, d_a, k):
        g = {kk: np.asarray(v, dtype=F32) for kk, v in sd.items()}
        self.norm_w, self.wq, self.keys1, self.keys2 = g["norm.w"], g["wq.weight"], g["keys1"], g["keys2"]
        self.values, self.log_scale, self.wo = g["values"], g["log_scale"], g["wo.weight"]
        self.d = self.wo.shape[0]
        self.h, self.n_sub, self.d_a, self.k = heads, n_sub, d_a, k
        self.dh, self.M = self.d // heads, n_sub * n_sub


def trained_sdm(p, x, bf16_stream=False, margins=True, force_si=None):
    """TrainedSdm.address + forward (M:438-457): q = wq RMSNorm(x); product-key top-k; softmax; weighted sum of
    the picked value rows (embedding_bag, sum mode); wo.  Returns (out, si, margin).  force_si (B*T, h, k): slot
    ids to use instead of the oracle's own (teacher forcing)."""
    B, T, _ = x.shape
    q = linear(rmsnorm(x, p.norm_w, bf16_stream=bf16_stream).reshape(B * T, p.d), p.wq).reshape(B * T, p.h, p.d_a)
    if margins:
        sv, si, margin = pk_address(q, p.keys1, p.keys2, p.k, return_margin=True, force_si=force_si)
    else:
        (sv, si), margin = pk_address(q, p.keys1, p.keys2, p.k, force_si=force_si), None
    w = softmax((sv * np.exp(p.log_scale)[None, :, None]).astype(F32, copy=False))
    r = np.zeros((B * T, p.h, p.dh), F32)
    for j in range(si.shape[-1]):
        r += w[..., j, None] * p.values[np.arange(p.h)[None, :], si[..., j]]
    out = linear(r.reshape(B, T, p.d), p.wo, bf16_out=bf16_stream)
    return out, si, margin


def swiglu(h, wg, wu, wd, bf16_stream=False):
    """SwiGLU.forward (L:96-97): down(silu(gate h) * up h), each bf16 op rounding in a bf16 stream."""
    g = linear(h, wg, bf16_out=bf16_stream)
    u = linear(h, wu, bf16_out=bf16_stream)
    s = silu(g)
    if bf16_stream:
        s = bf16(s)
        p = bf16(s * u)
    else:
        p = (s * u).astype(F32, copy=False)
    return linear(p, wd, bf16_out=bf16_stream)


def add_stream(x, y, bf16_stream):
    s = (x + y).astype(F32, copy=False)
    return bf16(s) if bf16_stream else s


def lm_forward(P, idx, bf16_stream=True, chunk=128, reset_at_bos=False, bos_id=0, collect=False, margins=True):
    """OneSdmLM.forward (M:525-555): enfold, L x (RunTimeSdm, then SwiGLU(RMSNorm) or TrainedSdm), nf, tied
    logits.  P is a dict: emb (V, d), nf_w (d,), layers: list of dicts with 'mem' (RunTimeSdmParams) and either
    'mlp' = (mnorm_w, wg, wu, wd) or 'sdm' (TrainedSdmParams).  Returns logits (B, T, V) and, with collect, the
    per-layer residual inputs and selections."""
    x = P["emb"][idx].astype(F32, copy=False)
    reset = (idx == bos_id) if reset_at_bos else None
    trace = []
    for lay in P["layers"]:
        rec = {"x_in": x}
        m_out, prep = rt_forward(lay["mem"], x, chunk=chunk, reset=reset, bf16_stream=bf16_stream, margins=margins)
        x = add_stream(x, m_out, bf16_stream)
        rec["prep"] = prep
        rec["x_mid"] = x
        if "mlp" in lay:
            nw, wg, wu, wd = lay["mlp"]
            x = add_stream(x, swiglu(rmsnorm(x, nw, bf16_stream=bf16_stream), wg, wu, wd, bf16_stream), bf16_stream)
        else:
            s_out, si, margin = trained_sdm(lay["sdm"], x, bf16_stream, margins)
            rec["sdm_si"], rec["sdm_margin"] = si, margin
            x = add_stream(x, s_out, bf16_stream)
        trace.append(rec)
    h = rmsnorm(x, P["nf_w"], bf16_stream=bf16_stream)
    logits = linear(h, P["emb"], bf16_out=bf16_stream)
    if collect:
        return logits, h, trace
    return logits


def ce_sum(logits, targets):
    """Sum over positions of cross-entropy (logsumexp - target logit).  The max-shifted exponentials are taken in
    float32 (each within about 1e-7 relative; numpy's float64 exp is scalar and ~50x slower), their sums, logs and
    the total in float64."""
    lg = logits.astype(F32, copy=False).reshape(-1, logits.shape[-1])
    m = lg.max(-1, keepdims=True)
    e = np.exp(lg - m).sum(-1, dtype=np.float64)
    lse = m[:, 0].astype(np.float64) + np.log(e)
    tl = lg[np.arange(lg.shape[0]), targets.reshape(-1)].astype(np.float64)
    return float((lse - tl).sum())


def matched_sdm_n_sub(d, mlp_f, heads, d_a):
    """matched_sdm_n_sub (M:465-468): the n_sub whose TrainedSdm weight count is closest to one SwiGLU + norm."""
    def params(n):
        return d + d * heads * d_a + heads * n * d_a + heads * n * n * (d // heads) + heads + d * d
    target = 3 * d * mlp_f + d
    return min(range(2, 4097), key=lambda n: abs(params(n) - target))
