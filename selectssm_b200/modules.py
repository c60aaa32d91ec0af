"""SelectiveSSM and BidirectionalMamba with the reference's fields and parameter names.

Mirrors ``SelectiveSSM`` (src/selectssm/selectssm.py:112-254) and
``BidirectionalMamba`` (src/selectssm/selectssm.py:256-364).  The dense
projections and norms stay in PyTorch (cuBLAS) -- they sit outside the graft,
as they sat in XLA in the reference.  The hot path -- flip/complement + causal
depthwise conv + activation, softplus(dt + bias), the selective scan, the D
skip and the gate -- runs in the sm_100a kernels behind the C ABI.

Parameters carry Flax's names and layouts, so a Flax parameter tree loads with
:meth:`load_flax_params`:

  SelectiveSSM:  shift_conv/kernel (K,1,D), A_log (D,N), BC/kernel (D,2N),
                 BC/bias (2N,), D (D,), dt/kernel (D,R), dt/bias (R,),
                 dt_proj/kernel (R,D), dt_proj/bias (D,)
  BidirectionalMamba: RMSNorm_0/scale (or LayerNorm_0/..., BatchNorm_0/...,
                 GroupNorm_0/...), in_proj/{kernel,bias}, ssm_fwd/..., ssm_rev/...,
                 out_proj/{kernel,bias}, mlp/..., mlp_proj/...

Flax creates parameters lazily from the first input; a torch module needs the
feature width up front, passed as ``features``.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import ops


# ----------------------------------------------------------------------------- initialisers
def _lecun_normal_(t: torch.Tensor, fan_in: int, generator=None) -> torch.Tensor:
    """Flax's lecun_normal: truncated normal (+-2 sd) with variance 1/fan_in."""
    std = math.sqrt(1.0 / fan_in) / 0.87962566103423978
    with torch.no_grad():
        nn.init.trunc_normal_(t, 0.0, 1.0, -2.0, 2.0, generator=generator)
        t.mul_(std)
    return t


def _inverse_softplus(x: torch.Tensor) -> torch.Tensor:
    """selectssm.py:16-17."""
    return x + torch.log(-torch.expm1(-x))


class _Dense(nn.Module):
    """flax.linen.Dense: y = x @ kernel + bias with kernel (in, out)."""

    def __init__(self, fin, fout, use_bias=True, bias_init=None, generator=None):
        super().__init__()
        self.kernel = nn.Parameter(_lecun_normal_(torch.empty(fin, fout), fin, generator))
        if use_bias:
            b = torch.zeros(fout) if bias_init is None else bias_init(fout)
            self.bias = nn.Parameter(b)
        else:
            self.register_parameter("bias", None)

    def forward(self, x):
        y = torch.matmul(x, self.kernel.to(x.dtype))
        return y if self.bias is None else y + self.bias.to(x.dtype)


def _act(x, name):
    if name == "silu":
        return F.silu(x)
    if name == "gelu":
        return F.gelu(x, approximate="tanh")  # flax nn.gelu default
    if name == "relu":
        return F.relu(x)
    if name is None:
        return x
    raise Exception(f"Unknown activation: {name}")


# ----------------------------------------------------------------------------- SelectiveSSM
class SelectiveSSM(nn.Module):
    """A variation on MAMBA: https://arxiv.org/pdf/2312.00752.pdf (selectssm.py:112-254).

    Fields as in the reference; ``features`` is the input width D.  The scan
    selector fields keep their meaning for validation (``chunk_size`` and
    ``n_channel_groups`` raise the reference's ValueErrors) while every
    selector runs the same CUDA kernels.
    """

    def __init__(self, features: int, reverse: bool = False, complement: bool = False, hidden_features: int = 16,
                 chunk_size: int = None, n_channel_groups: int = None, dt_rank="auto", dt_proj: bool = True,
                 dt_min: float = 0.001, dt_max: float = 0.1, regularize: bool = True, shift_l2_scale: float = 1e-7,
                 ssm_l2_scale: float = 1e-6, shift_conv_size: int = 3, activation: str = "silu",
                 diagnostics: dict = None, recursive_scan: bool = False, min_recursion_length: int = 2,
                 recursive_split: int = 2, custom_vjp_scan: bool = False, generator=None):
        super().__init__()
        D, N = features, hidden_features
        self.features, self.reverse, self.complement = D, reverse, complement
        self.hidden_features, self.chunk_size, self.n_channel_groups = N, chunk_size, n_channel_groups
        self.dt_rank = math.ceil(D / 16) if dt_rank == "auto" else dt_rank       # :158-161
        self.use_dt_proj, self.dt_min, self.dt_max = dt_proj, dt_min, dt_max
        self.regularize, self.shift_l2_scale, self.ssm_l2_scale = regularize, shift_l2_scale, ssm_l2_scale
        self.shift_conv_size, self.activation = shift_conv_size, activation
        self.diagnostics = dict(diagnostics or {})
        self.recursive_scan, self.min_recursion_length = recursive_scan, min_recursion_length
        self.recursive_split, self.custom_vjp_scan = recursive_split, custom_vjp_scan
        if activation not in ("silu", "gelu", "relu", None):
            raise Exception(f"Unknown activation: {activation}")                # :187
        R = self.dt_rank

        def dt_bias_init(n):                                                     # :194
            u = torch.empty(n).uniform_(dt_min, dt_max, generator=generator)
            return _inverse_softplus(u)

        self.shift_conv = nn.Module()
        self.shift_conv.kernel = nn.Parameter(
            _lecun_normal_(torch.empty(shift_conv_size, 1, D), shift_conv_size, generator))   # :170-174
        self.A_log = nn.Parameter(torch.log(torch.arange(1, N + 1, dtype=torch.float32)).repeat(D, 1))  # :190
        self.BC = _Dense(D, 2 * N, generator=generator)                          # :191
        self.D = nn.Parameter(torch.ones(D))                                     # :192
        self.dt = _Dense(D, R, bias_init=None if dt_proj else dt_bias_init, generator=generator)   # :195-197
        if dt_proj:
            self.dt_proj = _Dense(R, D, bias_init=dt_bias_init, generator=generator)              # :204
        elif R > 1 and D % R != 0:
            raise ValueError(f"dt_rank={R} must divide D={D}")                   # :207-208
        self.sown = {}  # values the reference sows into "diagnostics" / "losses"

    def _check_selector(self, L):
        if not (self.custom_vjp_scan or self.recursive_scan):
            ops._check_chunked(L, self.features, self.chunk_size, self.n_channel_groups)  # :47-54

    def scan_inputs(self, x):
        """The preamble up to the scan: (u, delta_raw, A, B, C, delta_bias) in the
        scan frame (selectssm.py:167-210); delta_raw excludes the dt_proj bias,
        which the scan kernel adds before its softplus."""
        B_, L, D = x.shape
        N = self.hidden_features
        self._check_selector(L)
        if "ssm_input_norm" in self.diagnostics:
            self.sown["ssm_input_mean"], self.sown["ssm_input_sd"] = x.mean(), x.std()
        u = ops.conv1d_act(x, self.shift_conv.kernel, self.activation, self.reverse, self.complement)
        A = -torch.exp(self.A_log)
        BC = self.BC(u)
        Bm, Cm = BC[..., :N], BC[..., N:]
        dt = self.dt(u)
        if self.use_dt_proj:
            delta, bias = torch.matmul(dt, self.dt_proj.kernel.to(dt.dtype)), self.dt_proj.bias
        else:
            R = self.dt_rank
            delta = dt.repeat_interleave(D // R, dim=-1) if R > 1 else dt.expand(B_, L, D)
            bias = None
        if "ssm_coeffs" in self.diagnostics:
            self.sown.update(activated_conv_mean=u.mean(), activated_conv_sd=u.std(), A_mean=A.mean(),
                             A_sd=A.std(), B_sd=Bm.std(), C_sd=Cm.std())
        return u, delta, A, Bm, Cm, bias

    def regularizer(self):
        """selectssm.py:241-248."""
        ks = [self.BC.kernel, self.dt.kernel] + ([self.dt_proj.kernel] if self.use_dt_proj else [])
        return (self.shift_l2_scale * (self.shift_conv.kernel ** 2).sum()
                + self.ssm_l2_scale * sum((k ** 2).sum() for k in ks))

    def forward(self, x, train: bool = False, z=None, gate_act="silu"):
        """x: (B, L, D).  Returns y + u*D (selectssm.py:230-238); with ``z`` the
        BidirectionalMamba gate y*act(z) is fused in as well."""
        u, delta, A, Bm, Cm, bias = self.scan_inputs(x)
        y = ops.selective_scan(u, delta, A, Bm, Cm, D=self.D, z=z, delta_bias=bias, delta_softplus=True,
                               reverse=self.reverse, complement=self.complement, gate_act=gate_act)
        if self.regularize:
            self.sown["ssm_regularizer"] = self.regularizer()
        if "ssm_output_norm" in self.diagnostics:
            self.sown["ssm_output_mean"], self.sown["ssm_output_sd"] = y.mean(), y.std()
        return y

    def forward_rc(self, x, train: bool = False):
        """rc(self(rc(x))) with rc(x)[b, l, d] = x[b, L-1-l, D-1-d]: the antisense
        strand of an RCPS wrapper (rcps.py:42-72), computed without flipping
        anything in memory.  The reversed, complemented read of the conv and
        scan kernels takes the place of the input flip, their unflipped store
        takes the place of the output flip, and the skip stays in the scan
        frame.  Only for a forward (reverse=False, complement=False) module."""
        if self.reverse or self.complement:
            raise ValueError("forward_rc needs a module with reverse=False and complement=False")
        self.reverse, self.complement = True, True
        try:
            u, delta, A, Bm, Cm, bias = self.scan_inputs(x)
        finally:
            self.reverse, self.complement = False, False
        y = ops.selective_scan(u, delta, A, Bm, Cm, D=self.D, delta_bias=bias, delta_softplus=True,
                               reverse=True, complement=True, aligned_skip=True)
        if self.regularize:
            self.sown["ssm_regularizer"] = self.regularizer()
        return y

    # ---- Flax parameter trees
    def load_flax_params(self, tree):
        """Copy a Flax SelectiveSSM parameter dict (numpy or torch arrays)."""
        def cp(param, arr):
            with torch.no_grad():
                param.copy_(torch.as_tensor(np.asarray(arr), dtype=param.dtype))
        cp(self.shift_conv.kernel, tree["shift_conv"]["kernel"])
        cp(self.A_log, tree["A_log"])
        cp(self.BC.kernel, tree["BC"]["kernel"]), cp(self.BC.bias, tree["BC"]["bias"])
        cp(self.D, tree["D"])
        cp(self.dt.kernel, tree["dt"]["kernel"]), cp(self.dt.bias, tree["dt"]["bias"])
        if self.use_dt_proj:
            cp(self.dt_proj.kernel, tree["dt_proj"]["kernel"]), cp(self.dt_proj.bias, tree["dt_proj"]["bias"])
        return self

    def flax_params(self):
        t = {"shift_conv": {"kernel": self.shift_conv.kernel}, "A_log": self.A_log,
             "BC": {"kernel": self.BC.kernel, "bias": self.BC.bias}, "D": self.D,
             "dt": {"kernel": self.dt.kernel, "bias": self.dt.bias}}
        if self.use_dt_proj:
            t["dt_proj"] = {"kernel": self.dt_proj.kernel, "bias": self.dt_proj.bias}
        return t


# ----------------------------------------------------------------------------- BidirectionalMamba
class _RMSNorm(nn.Module):
    """flax.linen.RMSNorm (epsilon 1e-6, learned scale)."""

    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.scale, self.eps = nn.Parameter(torch.ones(d)), eps

    def forward(self, x):
        xf = x.float()
        y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.scale
        return y.to(x.dtype)


class _LayerNorm(nn.Module):
    """flax.linen.LayerNorm (epsilon 1e-6, scale and bias)."""

    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.scale, self.bias, self.eps = nn.Parameter(torch.ones(d)), nn.Parameter(torch.zeros(d)), eps

    def forward(self, x):
        return F.layer_norm(x, x.shape[-1:], self.scale.to(x.dtype), self.bias.to(x.dtype), self.eps)


class _GroupNorm(nn.Module):
    """flax.linen.GroupNorm (num_groups 32, epsilon 1e-6) over the channel axis."""

    def __init__(self, d, groups=32, eps=1e-6):
        super().__init__()
        self.groups = math.gcd(groups, d) if d % groups else groups
        self.scale, self.bias, self.eps = nn.Parameter(torch.ones(d)), nn.Parameter(torch.zeros(d)), eps

    def forward(self, x):  # statistics over (L, channels-in-group) per batch row
        B_, L, D = x.shape
        xg = x.float().reshape(B_, L, self.groups, D // self.groups)
        mean = xg.mean(dim=(1, 3), keepdim=True)
        var = xg.var(dim=(1, 3), keepdim=True, unbiased=False)
        y = ((xg - mean) * torch.rsqrt(var + self.eps)).reshape(B_, L, D)
        return (y * self.scale + self.bias).to(x.dtype)


class _BatchNorm(nn.Module):
    """flax.linen.BatchNorm over (B, L) with Flax's momentum convention."""

    def __init__(self, d, momentum=0.9, eps=1e-5):
        super().__init__()
        self.bn = nn.BatchNorm1d(d, momentum=1.0 - momentum, eps=eps)

    def forward(self, x, train):
        self.bn.train(train)
        return self.bn(x.transpose(1, 2)).transpose(1, 2)


class BidirectionalMamba(nn.Module):
    """selectssm.py:256-364: norm -> in_proj -> forward and reverse SelectiveSSM
    -> gate (concatenated or summed) -> out_proj -> residual (-> MLP).

    With ``concatenate_fwd_rev`` both SSM scans, their D skips and the gates run
    in one kernel launch writing the concatenated (B, L, 2*ED) result."""

    def __init__(self, features: int, hidden_features: int, expansion_factor: float, dt_rank="auto",
                 complement: bool = False, tie_in_proj: bool = False, tie_gate: bool = False,
                 concatenate_fwd_rev: bool = True, activation: str = "silu", norm_type: str = "rms",
                 bn_momentum: float = 0.9, mlp_layer: bool = False, dense_expansion: int = 2,
                 mlp_dropout_rate: float = 0.1, ssm_args: dict = None, diagnostics: dict = None, generator=None):
        super().__init__()
        Din = features
        self.features, self.hidden_features, self.expansion_factor = Din, hidden_features, expansion_factor
        self.dt_rank = math.ceil(Din / 16) if dt_rank == "auto" else dt_rank   # :286-289
        self.complement, self.tie_in_proj, self.tie_gate = complement, tie_in_proj, tie_gate
        self.concatenate_fwd_rev, self.activation, self.norm_type = concatenate_fwd_rev, activation, norm_type
        self.mlp_layer, self.dense_expansion, self.mlp_dropout_rate = mlp_layer, dense_expansion, mlp_dropout_rate
        self.diagnostics = dict(diagnostics or {})
        if activation not in ("gelu", "silu", "relu"):
            raise Exception(f"Unknown activation: {activation}")               # :291-298
        ED = math.ceil(expansion_factor * Din)                                  # :315
        self.ED = ED
        norms = {"rms": ("RMSNorm_0", lambda: _RMSNorm(Din)), "layer": ("LayerNorm_0", lambda: _LayerNorm(Din)),
                 "group": ("GroupNorm_0", lambda: _GroupNorm(Din)),
                 "batch": ("BatchNorm_0", lambda: _BatchNorm(Din, bn_momentum))}
        self.norm_name = None
        if norm_type in norms:
            self.norm_name, mk = norms[norm_type]
            self.add_module(self.norm_name, mk())
        n_in = 1 if tie_in_proj else 2
        n_gate = 1 if tie_gate else 2
        self.in_proj = _Dense(Din, (n_in + n_gate) * ED, generator=generator)   # :319
        args = dict(ssm_args or {})
        self.ssm_fwd = SelectiveSSM(ED, hidden_features=hidden_features, reverse=False, dt_rank=self.dt_rank,
                                    diagnostics=self.diagnostics, generator=generator, **args)      # :325
        self.ssm_rev = SelectiveSSM(ED, hidden_features=hidden_features, reverse=True, complement=complement,
                                    dt_rank=self.dt_rank, diagnostics=self.diagnostics, generator=generator,
                                    **args)                                                             # :326
        self.out_proj = _Dense(2 * ED if concatenate_fwd_rev else ED, Din, generator=generator)         # :345
        if mlp_layer:
            self.mlp = _Dense(Din, dense_expansion * Din, generator=generator)                          # :357
            self.mlp_proj = _Dense(dense_expansion * Din, Din, generator=generator)                     # :360
        self.sown = {}

    def forward(self, x, train: bool = False):
        skip = x                                                                 # :300
        base = None
        if self.norm_type == "rms":  # one kernel: the norm and the residual base skip + out_proj.bias
            nm = getattr(self, self.norm_name)
            x, base = ops.rmsnorm_residual(x, nm.scale, self.out_proj.bias, nm.eps)
        elif self.norm_name is not None:
            nm = getattr(self, self.norm_name)
            x = nm(x, train) if self.norm_type == "batch" else nm(x)
        ED = self.ED
        n_in = 1 if self.tie_in_proj else 2
        proj = self.in_proj(x)
        xf = proj[..., :ED]
        xr = xf if self.tie_in_proj else proj[..., ED:2 * ED]                   # :320
        zf = proj[..., n_in * ED:(n_in + 1) * ED]
        zr = zf if self.tie_gate else proj[..., (n_in + 1) * ED:(n_in + 2) * ED]  # :321
        sf, sr = self.ssm_fwd, self.ssm_rev
        if self.concatenate_fwd_rev:                                             # :335-336, one launch
            uf, df, Af, Bf, Cf, bf = sf.scan_inputs(xf)
            ur, dr, Ar, Br, Cr, br = sr.scan_inputs(xr)
            g = ops.selective_scan_bidir(uf, df, Af, Bf, Cf, sf.D, bf, zf, ur, dr, Ar, Br, Cr, sr.D, br, zr,
                                         complement=self.complement, gate_act=self.activation)
            for m in (sf, sr):
                if m.regularize:
                    m.sown["ssm_regularizer"] = m.regularizer()
        else:                                                                    # :338
            g = sf(xf, train, z=zf, gate_act=self.activation) + sr(xr, train, z=zr, gate_act=self.activation)
        if "gated" in self.diagnostics and train:
            self.sown["gated_mean"], self.sown["gated_sd"] = g.mean(), g.std()
        if base is not None:                                                     # :345-352
            x = ops.dense_onto(base, g, self.out_proj.kernel)  # base + g W: GEMM with the residual as accumulator
        else:
            x = skip + self.out_proj(g)
        if self.mlp_layer:                                                       # :355-362
            skip = x
            h = F.dropout(self.mlp(x), self.mlp_dropout_rate, training=train)
            h = _act(h, self.activation)
            h = F.dropout(self.mlp_proj(h), self.mlp_dropout_rate, training=train)
            x = skip + h
        return x

    def load_flax_params(self, tree):
        """Copy a Flax BidirectionalMamba parameter dict (numpy or torch arrays)."""
        def cp(param, arr):
            with torch.no_grad():
                param.copy_(torch.as_tensor(np.asarray(arr), dtype=param.dtype))
        if self.norm_name is not None and self.norm_name in tree:
            nm = getattr(self, self.norm_name)
            for k, v in tree[self.norm_name].items():
                target = nm.bn.weight if (self.norm_type == "batch" and k == "scale") else \
                    nm.bn.bias if self.norm_type == "batch" else getattr(nm, k)
                cp(target, v)
        for name in ("in_proj", "out_proj") + (("mlp", "mlp_proj") if self.mlp_layer else ()):
            mod = getattr(self, name)
            cp(mod.kernel, tree[name]["kernel"])
            if mod.bias is not None:
                cp(mod.bias, tree[name]["bias"])
        self.ssm_fwd.load_flax_params(tree["ssm_fwd"])
        self.ssm_rev.load_flax_params(tree["ssm_rev"])
        return self
