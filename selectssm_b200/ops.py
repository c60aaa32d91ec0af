"""Scan operators over device tensors, with the reference's names and errors.

PyTorch is used here only as plumbing: device memory, the current CUDA stream
and autograd bookkeeping.  All arithmetic of the hot path runs in the sm_100a
kernels of ``libselectssm_b200.so``, reached through the C ABI (``_lib``).

Reference functions mirrored (paths within ihh/selectssm):

* :func:`ssm_chunked_scan`   src/selectssm/selectssm.py:37-109
* :func:`ssm_recursive_scan` src/selectssm/ssmrecscan.py:36-77
* :func:`ssm_scan`           src/selectssm/ssmrecscan.py:80-183 (custom VJP)

All three compute the same recurrence; their chunking arguments are memory
knobs in the reference with no numeric effect beyond rounding, so here they are
validated exactly as the reference validates them and then ignored.  The
extended op :func:`selective_scan` adds the softplus(dt + bias) preamble
(selectssm.py:204-210), the D skip (:238), the reverse/complement unflip
(:230-231) and the gate of BidirectionalMamba (:335-338).
"""

from __future__ import annotations

import torch

from . import _lib
from ._checks import check_chunked as _check_chunked, largest_factor_up_to  # noqa: F401

__all__ = [
    "selective_scan", "selective_scan_bidir", "ssm_chunked_scan", "ssm_recursive_scan", "ssm_scan",
    "conv1d_act", "largest_factor_up_to",
]


# ----------------------------------------------------------------------------- helpers
_DT = {torch.float32: _lib.SSM_F32, torch.bfloat16: _lib.SSM_BF16}


def _dtype_code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; the kernels take float32 or bfloat16") from None


def _ptr(t):
    return None if t is None else t.data_ptr()


def _rows(t: torch.Tensor, width: int):
    """(tensor, row stride) with unit stride along the last dim, (B,L,.) row-major
    rows and 16-byte alignment; copies only when the view does not qualify."""
    if t.dim() != 3:
        raise ValueError(f"expected a (batch, seqlen, features) tensor, got shape {tuple(t.shape)}")
    es = t.element_size()
    ok = (t.stride(2) == 1 and t.shape[2] == width and t.stride(0) == t.shape[1] * t.stride(1)
          and t.data_ptr() % 16 == 0 and (t.stride(1) * es) % 16 == 0)
    if not ok:
        t = t.contiguous()
    return t, t.stride(1)


def _dense(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() and t.data_ptr() % 16 == 0 else t.contiguous()


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("selectssm_b200 ops run on CUDA tensors only (no CPU fallback)")


def _flags(delta_softplus, reverse, complement, aligned_skip):
    f = 0
    if delta_softplus:
        f |= _lib.SSM_DELTA_SOFTPLUS
    if reverse:
        f |= _lib.SSM_REVERSE
        if complement:
            f |= _lib.SSM_COMPLEMENT
    if aligned_skip:
        f |= _lib.SSM_ALIGNED_SKIP
    return f


class _Prepared:
    """Validated, layout-normalised arguments of one scan direction."""

    def __init__(self, u, delta, A, B, C, D, z, delta_bias, delta_softplus, reverse, complement, gate_act,
                 aligned_skip):
        _require_cuda(u, delta, A, B, C, D, z, delta_bias)
        if u.dim() != 3:
            raise ValueError(f"u must be (batch, seqlen, dim), got {tuple(u.shape)}")
        Bsz, L, Dm = u.shape
        N = A.shape[-1]
        if A.shape != (Dm, N):
            raise ValueError(f"A must be (dim, dstate) = ({Dm}, {N}), got {tuple(A.shape)}")
        if N != _lib.DSTATE:
            raise ValueError(f"dstate (hidden_features) must be {_lib.DSTATE} for this build, got {N}")
        if delta.shape != u.shape:
            if delta.dim() == 3 and delta.shape[:2] == u.shape[:2] and delta.shape[2] == 1:
                delta = delta.expand(Bsz, L, Dm)  # the reference broadcasts (B,L,1)
            else:
                raise ValueError(f"delta must be {tuple(u.shape)} or (B,L,1), got {tuple(delta.shape)}")
        for name, t in (("B", B), ("C", C)):
            if t.shape != (Bsz, L, N):
                raise ValueError(f"{name} must be ({Bsz}, {L}, {N}), got {tuple(t.shape)}")
        if z is not None and z.shape != u.shape:
            raise ValueError(f"z must match u {tuple(u.shape)}, got {tuple(z.shape)}")
        self.dtype = u.dtype
        _dtype_code(u)
        if B.dtype != C.dtype:
            raise ValueError("B and C must share a dtype")
        self.u = _dense(u)
        self.delta = _dense(delta.to(u.dtype))
        self.A = _dense(A.float())
        B, self.bc_stride = _rows(B, N)
        C2, cs = _rows(C, N)
        if cs != self.bc_stride:
            B, C2 = B.contiguous(), C2.contiguous()
            self.bc_stride = N
        self.B, self.C = B, C2
        self.D = None if D is None else _dense(D.float())
        self.delta_bias = None if delta_bias is None else _dense(delta_bias.float())
        if z is not None:
            z, self.z_stride = _rows(z.to(u.dtype), Dm)
        else:
            self.z_stride = 0
        self.z = z
        if (Dm * u.element_size()) % 16:
            raise ValueError(f"dim={Dm} must be a multiple of {16 // u.element_size()} for {u.dtype}")
        self.shape = (Bsz, L, Dm)
        self.flags = _flags(delta_softplus, reverse, complement, aligned_skip)
        self.gate_act = _lib.ACT_CODES[gate_act] if z is not None else 0
        self.reverse, self.complement = reverse, complement

    def params(self, out=None, out_stride=0, states=None) -> _lib.SSMParams:
        Bsz, L, Dm = self.shape
        p = _lib.SSMParams()
        p.batch, p.seqlen, p.dim, p.dstate = Bsz, L, Dm, _lib.DSTATE
        p.dtype = _dtype_code(self.u)
        p.bc_dtype = _dtype_code(self.B)
        p.flags = self.flags
        p.gate_act = self.gate_act
        p.z_stride = self.z_stride
        p.out_stride = out_stride
        p.bc_stride = self.bc_stride
        p.u, p.delta, p.A = _ptr(self.u), _ptr(self.delta), _ptr(self.A)
        p.Bm, p.Cm, p.D = _ptr(self.B), _ptr(self.C), _ptr(self.D)
        p.delta_bias, p.z = _ptr(self.delta_bias), _ptr(self.z)
        p.out, p.states = _ptr(out), _ptr(states)
        return p

    def new_states(self) -> torch.Tensor:
        Bsz, L, Dm = self.shape
        nblk = (L + _lib.SSM_CHUNK - 1) // _lib.SSM_CHUNK
        return torch.empty((Bsz, nblk, Dm, _lib.DSTATE), dtype=torch.float32, device=self.u.device)

    def grads(self, p: _lib.SSMParams, dout, dout_stride):
        """Allocate gradient buffers and fill the backward fields of ``p``."""
        Bsz, L, Dm = self.shape
        dev = self.u.device
        g = {
            "du": torch.empty_like(self.u),
            "ddelta": torch.empty_like(self.u),
            "dA": torch.empty((Dm, _lib.DSTATE), dtype=torch.float32, device=dev),
            "dB": torch.empty((Bsz, L, _lib.DSTATE), dtype=self.B.dtype, device=dev),
            "dC": torch.empty((Bsz, L, _lib.DSTATE), dtype=self.C.dtype, device=dev),
            "dD": None if self.D is None else torch.empty(Dm, dtype=torch.float32, device=dev),
            "ddelta_bias": None if self.delta_bias is None else torch.empty(Dm, dtype=torch.float32, device=dev),
            "dz": None if self.z is None else torch.empty((Bsz, L, Dm), dtype=self.u.dtype, device=dev),
        }
        p.dout, p.out_stride = _ptr(dout), dout_stride
        p.du, p.ddelta, p.dA = _ptr(g["du"]), _ptr(g["ddelta"]), _ptr(g["dA"])
        p.dB, p.dC, p.dD = _ptr(g["dB"]), _ptr(g["dC"]), _ptr(g["dD"])
        p.ddelta_bias, p.dz = _ptr(g["ddelta_bias"]), _ptr(g["dz"])
        # dB/dC are written with the B/C row stride; keep them dense
        p.bc_stride = _lib.DSTATE if self.bc_stride != _lib.DSTATE else self.bc_stride
        if p.bc_stride != self.bc_stride:
            self.B, self.C = self.B.contiguous(), self.C.contiguous()
            p.Bm, p.Cm = _ptr(self.B), _ptr(self.C)
        # dz uses the z row stride: give it z's stride only when z is dense
        if self.z is not None and self.z_stride != Dm:
            self.z = self.z.contiguous()
            p.z, p.z_stride = _ptr(self.z), Dm
        return g


def _workspace(p: _lib.SSMParams, device, extra=None, kind=None) -> torch.Tensor:
    """Scratch for one call: ``kind`` "fwd", "bwd" or "bwd_mc" sizes it for
    that call alone; None for any call on these params (and ``extra``)."""
    lib = _lib.load()
    if kind == "fwd":
        n = lib.ssm_fwd_workspace_bytes(p)
    elif kind in ("bwd", "bwd_mc"):
        n = lib.ssm_bwd_workspace_bytes(p, int(kind == "bwd_mc"))
    else:
        n = lib.ssm_workspace_bytes(p) + (0 if extra is None else lib.ssm_workspace_bytes(extra))
    ws = torch.empty(max(n, 256), dtype=torch.uint8, device=device)
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    return ws


# ----------------------------------------------------------------------------- autograd
class _SelectiveScanFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, u, delta, A, B, C, D, z, delta_bias, delta_softplus, reverse, complement, gate_act,
                aligned_skip, bc_sum=None):
        pr = _Prepared(u, delta, A, B, C, D, z, delta_bias, delta_softplus, reverse, complement, gate_act,
                       aligned_skip)
        out = torch.empty(pr.shape, dtype=pr.dtype, device=pr.u.device)
        states = pr.new_states()
        p = pr.params(out=out, out_stride=pr.shape[2], states=states)
        ws = _workspace(p, pr.u.device, kind="fwd")  # segment carries, widened bf16 B / C
        _lib.check(_lib.load().ssm_fwd(ctypes_byref(p), _stream()), "ssm_fwd")
        del ws
        ctx.pr = pr
        ctx.bc_sum = bc_sum
        ctx.delta_broadcast = delta.shape[-1] == 1 and u.shape[-1] != 1
        ctx.save_for_backward(states)
        return out

    @staticmethod
    def backward(ctx, dout):
        (states,) = ctx.saved_tensors
        pr = ctx.pr
        dout = _dense(dout.to(pr.dtype))
        p = pr.params(states=states)
        g = pr.grads(p, dout, pr.shape[2])
        ws = _workspace(p, pr.u.device, kind="bwd" if ctx.bc_sum is None else "bwd_mc")
        if ctx.bc_sum is None:
            _lib.check(_lib.load().ssm_bwd(ctypes_byref(p), _stream()), "ssm_bwd")
        else:  # dB / dC summed over the channel shards inside the kernel
            mc = ctx.bc_sum.begin(pr.shape[0], pr.shape[1])
            _lib.check(_lib.load().ssm_bwd_bc_multicast(ctypes_byref(p), mc, _stream()), "ssm_bwd_bc_multicast")
            g["dB"], g["dC"] = ctx.bc_sum.end(pr.B.dtype)
        del ws
        ddelta = g["ddelta"]
        if ctx.delta_broadcast:
            ddelta = ddelta.sum(-1, keepdim=True)
        return (g["du"], ddelta, g["dA"], g["dB"], g["dC"], g["dD"], g["dz"], g["ddelta_bias"],
                None, None, None, None, None, None)


def ctypes_byref(p):
    import ctypes
    return ctypes.byref(p)


def selective_scan(u, delta, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False, reverse=False,
                   complement=False, gate_act="silu", aligned_skip=False, bc_sum=None):
    """Fused selective scan on CUDA tensors (differentiable).

    u, delta: (batch, L, dim) in the scan frame; A: (dim, 16) fp32; B, C:
    (batch, L, 16); D, delta_bias: (dim,); z: (batch, L, dim) in the output
    frame.  Returns ``(flip(y_scan) + skip) * act(z)`` where ``y_scan`` is the
    scan of dt = softplus(delta + delta_bias) (or delta + delta_bias).
    ``reverse``/``complement`` follow SelectiveSSM (selectssm.py:115-116, 167-168,
    230-231); the skip adds the scan-frame ``u * D`` unflipped, as the reference
    does at selectssm.py:238, unless ``aligned_skip``.

    ``bc_sum`` (a ``parallel.MulticastBCSum``) is for d_inner sharding with B
    and C replicated: the backward kernel then sums dB / dC over the group's
    ranks through NVLink multicast, so the returned B / C gradients are the
    totals (do not also wrap B, C in ``parallel.replicated_bc``).
    """
    return _SelectiveScanFn.apply(u, delta, A, B, C, D, z, delta_bias, bool(delta_softplus), bool(reverse),
                                  bool(complement), gate_act, bool(aligned_skip), bc_sum)


# ----------------------------------------------------------------------------- reference API
def ssm_chunked_scan(x, Acoeff, Bcoeff, Ccoeff, dt, chunk_size: int = None, n_channel_groups: int = 1):
    """Drop-in for selectssm.ssm_chunked_scan (selectssm.py:37-109).

    x, dt: (B, L, D) (dt may be (B, L, 1)); Acoeff: (D, N); Bcoeff, Ccoeff:
    (B, L, N).  Returns y (B, L, D) with y_t = C_t . h_t,
    h_t = exp(A dt_t) h_{t-1} + dt_t B_t x_t.  chunk_size / n_channel_groups are
    checked as the reference checks them; the kernel's own chunking replaces them.
    """
    _check_chunked(x.shape[-2], x.shape[-1], chunk_size, n_channel_groups)
    return selective_scan(x, dt, Acoeff, Bcoeff, Ccoeff)


def ssm_recursive_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, min_recursion_length: int = 2, recursive_split: int = 2):
    """Drop-in for selectssm.ssm_recursive_scan (ssmrecscan.py:36-77); same result
    as :func:`ssm_chunked_scan`."""
    if recursive_split < 1:
        raise ValueError(f"recursive_split={recursive_split} must be >= 1")
    return selective_scan(x, Delta, Acoeff, Bcoeff, Ccoeff)


def ssm_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, min_recursion_length: int = 2, recursive_split: int = 2):
    """Drop-in for selectssm.ssm_scan (ssmrecscan.py:80-83): the recursive scan
    with a hand-written backward; here both directions are the CUDA kernels and
    the backward returns (dx, dA, dB, dC, dDelta) like ssm_scan_backward (:163-181)."""
    return ssm_recursive_scan(x, Acoeff, Bcoeff, Ccoeff, Delta, min_recursion_length, recursive_split)


# ----------------------------------------------------------------------------- bidirectional
class _BidirScanFn(torch.autograd.Function):
    """Both SelectiveSSM directions of BidirectionalMamba in one launch, writing
    [y_f * act(z_f), y_r * act(z_r)] into one (B, L, 2*dim) buffer
    (concatenate_fwd_rev, selectssm.py:336)."""

    @staticmethod
    def forward(ctx, uf, df, Af, Bf, Cf, Df, biasf, zf, ur, dr, Ar, Br, Cr, Dr, biasr, zr, complement, gate_act,
                aligned_skip):
        prf = _Prepared(uf, df, Af, Bf, Cf, Df, zf, biasf, True, False, False, gate_act, aligned_skip)
        prr = _Prepared(ur, dr, Ar, Br, Cr, Dr, zr, biasr, True, True, complement, gate_act, aligned_skip)
        Bsz, L, Dm = prf.shape
        out = torch.empty((Bsz, L, 2 * Dm), dtype=prf.dtype, device=prf.u.device)
        sf, sr = prf.new_states(), prr.new_states()
        pf = prf.params(out=out[..., :Dm], out_stride=2 * Dm, states=sf)
        pr = prr.params(out=out[..., Dm:], out_stride=2 * Dm, states=sr)
        wsf, wsr = _workspace(pf, prf.u.device), _workspace(pr, prr.u.device)
        _lib.check(_lib.load().ssm_fwd_bidir(ctypes_byref(pf), ctypes_byref(pr), _stream()), "ssm_fwd_bidir")
        del wsf, wsr
        ctx.prs = (prf, prr)
        ctx.save_for_backward(sf, sr)
        return out

    @staticmethod
    def backward(ctx, dout):
        sf, sr = ctx.saved_tensors
        prf, prr = ctx.prs
        Dm = prf.shape[2]
        dout, ostride = _rows(dout.to(prf.dtype), 2 * Dm)
        pf, pr = prf.params(states=sf), prr.params(states=sr)
        gf = prf.grads(pf, dout[..., :Dm], ostride)
        gr = prr.grads(pr, dout[..., Dm:], ostride)
        ws = _workspace(pf, prf.u.device, extra=pr)
        _lib.check(_lib.load().ssm_bwd_bidir(ctypes_byref(pf), ctypes_byref(pr), _stream()), "ssm_bwd_bidir")
        del ws
        out = []
        for g in (gf, gr):
            out += [g["du"], g["ddelta"], g["dA"], g["dB"], g["dC"], g["dD"], g["ddelta_bias"], g["dz"]]
        return tuple(out) + (None, None, None)


def selective_scan_bidir(uf, delta_f, Af, Bf, Cf, Df, bias_f, zf, ur, delta_r, Ar, Br, Cr, Dr, bias_r, zr,
                         complement=False, gate_act="silu", aligned_skip=False):
    """Forward and reverse SelectiveSSM scans (softplus on, D skip, gate) in one
    launch; returns the concatenated gated output (B, L, 2*dim)."""
    return _BidirScanFn.apply(uf, delta_f, Af, Bf, Cf, Df, bias_f, zf, ur, delta_r, Ar, Br, Cr, Dr, bias_r, zr,
                              bool(complement), gate_act, bool(aligned_skip))


# ----------------------------------------------------------------------------- conv preamble
class _Conv1dActFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, act, reverse, complement):
        _require_cuda(x, w)
        Bsz, L, Dm = x.shape
        K = w.shape[0]
        w_shape = w.shape
        x, xs = _rows(x, Dm)
        w = _dense(w.float().reshape(K, Dm))
        u = torch.empty((Bsz, L, Dm), dtype=x.dtype, device=x.device)
        p = _conv_params(x, xs, w, act, reverse, complement)
        p.u = u.data_ptr()
        _lib.check(_lib.load().ssm_conv1d_act_fwd(ctypes_byref(p), _stream()), "ssm_conv1d_act_fwd")
        ctx.save_for_backward(x, w)
        ctx.cfg = (xs, act, reverse, complement)
        ctx.w_shape = w_shape
        return u

    @staticmethod
    def backward(ctx, du):
        x, w = ctx.saved_tensors
        xs, act, reverse, complement = ctx.cfg
        du = _dense(du.to(x.dtype))
        dx = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        dw = torch.empty_like(w)
        p = _conv_params(x, xs, w, act, reverse, complement)
        # dx is dense; x may be a strided view
        if xs != x.shape[2]:
            x = x.contiguous()
            p.x, p.x_stride = x.data_ptr(), x.shape[2]
        p.du, p.dx, p.dw = du.data_ptr(), dx.data_ptr(), dw.data_ptr()
        lib = _lib.load()
        ws = torch.empty(max(lib.ssm_conv1d_workspace_bytes(ctypes_byref(p)), 256), dtype=torch.uint8,
                         device=x.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.ssm_conv1d_act_bwd(ctypes_byref(p), _stream()), "ssm_conv1d_act_bwd")
        del ws
        return dx, dw.reshape(ctx.w_shape), None, None, None


def _conv_params(x, xs, w, act, reverse, complement):
    Bsz, L, Dm = x.shape
    p = _lib.SSMConvParams()
    p.batch, p.seqlen, p.dim, p.width = Bsz, L, Dm, w.shape[0]
    p.dtype = _dtype_code(x)
    p.flags = _flags(False, reverse, complement, False)
    p.act = _lib.ACT_CODES[act]
    p.x_stride = xs
    p.x, p.w = x.data_ptr(), w.data_ptr()
    return p


def conv1d_act(x, w, act="silu", reverse=False, complement=False):
    """u = act(causal depthwise conv(flip(x), w)) (selectssm.py:167-187).

    x: (B, L, D) in its own frame; w: Flax's ``shift_conv/kernel`` (K, 1, D) or
    (K, D).  u is in the scan frame (flipped when ``reverse``)."""
    return _Conv1dActFn.apply(x, w, act, bool(reverse), bool(complement))


# ----------------------------------------------------------------------------- RMSNorm + residual base
class _RMSNormResidualFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, scale, res_bias, eps):
        _require_cuda(x, scale)
        dim = x.shape[-1]
        x2 = _dense(x).reshape(-1, dim)
        scale = _dense(scale.float())
        y = torch.empty_like(x2)
        base = torch.empty_like(x2)
        rstd = torch.empty(x2.shape[0], dtype=torch.float32, device=x.device)
        p = _norm_params(x2, scale, eps, rstd)
        bias = None if res_bias is None else _dense(res_bias.float())
        p.y, p.res_base = y.data_ptr(), base.data_ptr()
        p.res_bias = 0 if bias is None else bias.data_ptr()
        _lib.check(_lib.load().ssm_rmsnorm_fwd(ctypes_byref(p), _stream()), "ssm_rmsnorm_fwd")
        ctx.save_for_backward(x2, scale, rstd)
        ctx.eps, ctx.shape, ctx.has_bias = eps, x.shape, res_bias is not None
        return y.view(x.shape), base.view(x.shape)

    @staticmethod
    def backward(ctx, dy, dbase):
        x2, scale, rstd = ctx.saved_tensors
        dim = x2.shape[1]
        dy = torch.zeros_like(x2) if dy is None else _dense(dy.to(x2.dtype)).reshape(-1, dim)
        dres = None if dbase is None else _dense(dbase.to(x2.dtype)).reshape(-1, dim)
        dx = torch.empty_like(x2)
        dscale = torch.empty(dim, dtype=torch.float32, device=x2.device)
        p = _norm_params(x2, scale, ctx.eps, rstd)
        p.dy, p.dx, p.dscale = dy.data_ptr(), dx.data_ptr(), dscale.data_ptr()
        p.dres = 0 if dres is None else dres.data_ptr()
        lib = _lib.load()
        ws = torch.empty(max(lib.ssm_rmsnorm_workspace_bytes(ctypes_byref(p)), 256), dtype=torch.uint8,
                         device=x2.device)
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.ssm_rmsnorm_bwd(ctypes_byref(p), _stream()), "ssm_rmsnorm_bwd")
        del ws
        dbias = None
        if ctx.has_bias:
            dbias = torch.zeros(dim, dtype=torch.float32, device=x2.device) if dres is None else dres.float().sum(0)
        return dx.view(ctx.shape), dscale, dbias, None


def _norm_params(x2, scale, eps, rstd):
    p = _lib.SSMNormParams()
    p.rows, p.dim = x2.shape[0], x2.shape[1]
    p.dtype = _dtype_code(x2)
    p.eps = float(eps)
    p.x, p.scale, p.rstd = x2.data_ptr(), scale.data_ptr(), rstd.data_ptr()
    return p


def rmsnorm_residual(x, scale, res_bias=None, eps=1e-6):
    """flax.linen.RMSNorm of x over its last axis (selectssm.py:306-313) and, in
    the same pass, the residual base x + res_bias of the block's output
    (selectssm.py:345-352, with out_proj's bias folded in).  Returns (y, base)."""
    return _RMSNormResidualFn.apply(x, scale, res_bias, float(eps))


def dense_onto(base, h, kernel):
    """base + h @ kernel in one cuBLAS call (the residual add of out_proj)."""
    d = kernel.shape[1]
    out = torch.addmm(base.reshape(-1, d), h.reshape(-1, h.shape[-1]), kernel.to(h.dtype))
    return out.view(*h.shape[:-1], d)
