"""CPU oracle for the PP-OCRv6 detector / recognizer forward passes.

TEST INFRASTRUCTURE ONLY.  This module restates, in FP32 on the CPU, the
arithmetic of the reference's native CPU backend (ppocr-rs src/cpu/model.rs,
src/cpu/backend.rs, src/cpu/ops.rs, src/cpu/kernels/mod.rs).  It is the
checker for the CUDA path: only tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline leg import it.  The product never calls into it.

Parity status: unpinned against execution of the reference.  The reference
cannot be compiled or run here (Rust toolchain absent, wgpu GPU path needs a
graphics API), so model-level parity rests on this restatement plus the
reference's own known-answer tests, which tests/test_oracle.py re-expresses
against these functions.

Convolutions use torch's CPU FP32 conv (exact FP32 products and sums, only
the summation order differs from the reference's packed AVX2 GEMMs); every
activation, fold and factorisation is written out as the reference states it.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch
import torch.nn.functional as F

torch.backends.mkldnn.enabled = True

Tensor = torch.Tensor

# ---------------------------------------------------------------------------
# Elementwise formulas (src/cpu/kernels/mod.rs:2365-2403)
# ---------------------------------------------------------------------------


def erf_as(x: Tensor) -> Tensor:
    """Abramowitz-Stegun 7.1.26 erf, as kernels/mod.rs:2393-2403 writes it."""
    sign = torch.where(x < 0, -1.0, 1.0).to(x.dtype)
    a = x.abs()
    t = 1.0 / (a * 0.3275911 + 1.0)
    poly = t * (0.2548296 + t * (-0.28449672 + t * (1.4214138 + t * (-1.4531521 + t * 1.0614054))))
    return sign * (1.0 - poly * torch.exp(-a * a))


def gelu(x: Tensor) -> Tensor:
    """0.5 x (1 + erf(x / sqrt 2)) with the A&S erf (kernels/mod.rs:2383)."""
    return 0.5 * x * (1.0 + erf_as(x * (1.0 / math.sqrt(2.0))))


def relu(x: Tensor) -> Tensor:
    return torch.clamp(x, min=0.0)


def silu(x: Tensor) -> Tensor:
    return x / (1.0 + torch.exp(-x))


def sigmoid(x: Tensor) -> Tensor:
    return 1.0 / (1.0 + torch.exp(-x))


def hard_swish(x: Tensor) -> Tensor:
    return x * torch.clamp(x / 6.0 + 0.5, 0.0, 1.0)


def hard_sigmoid(x: Tensor, alpha: float, beta: float) -> Tensor:
    return torch.clamp(x * alpha + beta, 0.0, 1.0)


ACTIVATIONS = {
    None: lambda x: x,
    "none": lambda x: x,
    "relu": relu,
    "silu": silu,
    "gelu": gelu,
    "hswish": hard_swish,
    "sigmoid": sigmoid,
}

# ---------------------------------------------------------------------------
# Weight access (src/cpu/weights.rs:13-95)
# ---------------------------------------------------------------------------


class Weights:
    """Name -> float32 tensor map with the reference's shape checks."""

    def __init__(self, tensors: Dict[str, np.ndarray]):
        self.tensors = {k: np.asarray(v, dtype=np.float32) for k, v in tensors.items()}

    @classmethod
    def load(cls, path: str) -> "Weights":
        from safetensors.numpy import load_file

        return cls(load_file(str(path)))

    def get(self, name: str, shape: Sequence[int]) -> np.ndarray:
        if name not in self.tensors:
            raise KeyError(f"missing tensor {name!r}")
        value = self.tensors[name]
        if tuple(value.shape) != tuple(shape):
            raise ValueError(f"tensor {name!r} expects shape {tuple(shape)}, found {value.shape}")
        return value


def fold_batch_norm(weight: np.ndarray, bias: Optional[np.ndarray], w: Weights, prefix: str, channels: int):
    """BN fold of cpu/model.rs:371-407: scale = g/sqrt(v+1e-5); W *= scale; b = (b-m)*scale+beta (f32)."""
    gamma = w.get(f"{prefix}.weight", (channels,))
    beta = w.get(f"{prefix}.bias", (channels,))
    mean = w.get(f"{prefix}.running_mean", (channels,))
    var = w.get(f"{prefix}.running_var", (channels,))
    scale = (gamma / np.sqrt(var + np.float32(1e-5))).astype(np.float32)
    out_w = (weight.reshape(channels, -1) * scale[:, None]).reshape(weight.shape).astype(np.float32)
    b = np.zeros(channels, np.float32) if bias is None else bias.astype(np.float32)
    out_b = ((b - mean) * scale + beta).astype(np.float32)
    return out_w, out_b


def fold_transpose_batch_norm(weight: np.ndarray, bias: np.ndarray, w: Weights, prefix: str, cout: int):
    """BN fold over the output axis of an IOHW transposed-conv weight (cpu/model.rs:1440-1477)."""
    gamma = w.get(f"{prefix}.weight", (cout,))
    beta = w.get(f"{prefix}.bias", (cout,))
    mean = w.get(f"{prefix}.running_mean", (cout,))
    var = w.get(f"{prefix}.running_var", (cout,))
    scale = (gamma / np.sqrt(var + np.float32(1e-5))).astype(np.float32)
    out_w = (weight * scale[None, :, None, None]).astype(np.float32)
    out_b = ((bias - mean) * scale + beta).astype(np.float32)
    return out_w, out_b


def factor_rank_one(weight: np.ndarray, cin: int, cout: int, k: int):
    """Rank-one split of an [O, I, k, k] kernel into depthwise [I, k*k] and pointwise [O, I].

    Power iteration (4 rounds, float64) per input channel, started from the
    output channel of largest energy, then the same acceptance test as
    cpu/model.rs:221-369 (max error <= 1e-5 * max|w| + 1e-12, relative
    Frobenius error <= 1e-6).
    """
    src = weight.reshape(cout, cin, k * k).astype(np.float64)
    src32 = weight.reshape(cout, cin, k * k)
    if not np.all(np.isfinite(src32)):
        raise ValueError("rank-one convolution weight contains non-finite values")
    depthwise = np.zeros((cin, k * k), np.float32)
    pointwise = np.zeros((cout, cin), np.float32)
    for i in range(cin):
        block = src[:, i, :]  # [O, k*k]
        energy = (block * block).sum(axis=1)
        o0 = int(np.argmax(energy)) if energy.max() > 0 else 0
        # first strictly-greater wins, as the reference's loop does
        best = 0.0
        o0 = 0
        for o in range(cout):
            if energy[o] > best:
                best = energy[o]
                o0 = o
        if best == 0.0:
            continue
        direction = block[o0] / math.sqrt(best)
        for _ in range(4):
            scales = block @ direction
            se = float((scales * scales).sum())
            if not (math.isfinite(se) and se > 0):
                raise ValueError("rank-one convolution factorization became degenerate")
            direction = (scales @ block) / se
            norm = math.sqrt(float((direction * direction).sum()))
            if not (math.isfinite(norm) and norm > 0):
                raise ValueError("rank-one convolution spatial factor became degenerate")
            direction = direction / norm
        scales = block @ direction
        pointwise[:, i] = scales.astype(np.float32)
        depthwise[i] = direction.astype(np.float32)
    recon = pointwise[:, :, None] * depthwise[None, :, :]
    err = np.abs(src32 - recon).astype(np.float64)
    max_src = float(np.abs(src32).max()) if src32.size else 0.0
    src_energy = float((src32.astype(np.float64) ** 2).sum())
    rel = 0.0 if src_energy == 0 else math.sqrt(float((err * err).sum()) / src_energy)
    limit = max_src * 1e-5 + 1e-12
    if not (float(err.max()) <= limit and rel <= 1e-6):
        raise ValueError(f"fused convolution is not rank-one separable: max error {err.max():.6e} "
                         f"(limit {limit:.6e}), relative Frobenius error {rel:.6e}")
    return depthwise.reshape(cin, 1, k, k), pointwise.reshape(cout, cin, 1, 1)


def fuse_intraclass(sym_w, sym_b, ver_w, ver_b, hor_w, hor_b):
    """Add the k x 1 and 1 x k branches into the centre column / row (cpu/model.rs:811-888)."""
    o, i, kh, kw = sym_w.shape
    if kh != kw or kh % 2 == 0:
        raise ValueError("intraclass symmetric kernel must be odd and square")
    if ver_w.shape != (o, i, kh, 1) or hor_w.shape != (o, i, 1, kw):
        raise ValueError("intraclass branch weight shape mismatch")
    c = kh // 2
    w = sym_w.astype(np.float32).copy()
    w[:, :, :, c] += ver_w[:, :, :, 0]
    w[:, :, c, :] += hor_w[:, :, 0, :]
    b = (sym_b.astype(np.float32) + ver_b) + hor_b
    return w, b.astype(np.float32)


# ---------------------------------------------------------------------------
# Operators (src/cpu/ops.rs)
# ---------------------------------------------------------------------------


_DTYPE = torch.float32


class compute_dtype:
    """Context manager: run the oracle's arithmetic in another dtype.

    ``with compute_dtype(torch.float64): ...`` evaluates the same graph, with
    the same (F32-folded) parameters, in double precision.  The distance
    between the float32 and float64 evaluations is the FP32 rounding noise of
    the network itself, which bounds how closely any FP32 implementation with
    a different summation order can agree with the reference.
    """

    def __init__(self, dtype):
        self.dtype = dtype

    def __enter__(self):
        global _DTYPE
        self.prev, _DTYPE = _DTYPE, self.dtype
        return self

    def __exit__(self, *exc):
        global _DTYPE
        _DTYPE = self.prev


# Optional capture of intermediate activations (test diagnostics only): while
# TRACE is a dict, the detector's modules store their outputs in it (NCHW)
# under the names the CUDA plan gives the same tensors.
TRACE: Optional[Dict[str, Tensor]] = None


def _trace(name: str, x: Tensor) -> Tensor:
    if TRACE is not None:
        TRACE[name] = x.detach().clone()
    return x


def t(a: np.ndarray) -> Tensor:
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(_DTYPE)


def conv2d(x: Tensor, weight: np.ndarray, bias: Optional[np.ndarray], stride=(1, 1),
           pads=(0, 0, 0, 0), groups: int = 1) -> Tensor:
    """NCHW conv; pads are [top, left, bottom, right] as in the reference's ConvOptions."""
    top, left, bottom, right = pads
    if any(pads):
        x = F.pad(x, (left, right, top, bottom))
    return F.conv2d(x, t(weight), None if bias is None else t(bias), stride=tuple(stride), groups=groups)


def max_pool_same_upper(x: Tensor) -> Tensor:
    # Note: in float64 mode F.pad keeps the dtype; -inf padding never wins.
    """2x2 stride-1 max pool padded at bottom/right; pads never win (ops.rs:1520-1535)."""
    x = F.pad(x, (0, 1, 0, 1), value=float("-inf"))
    return F.max_pool2d(x, kernel_size=2, stride=1)


def avg_pool_3x2(x: Tensor) -> Tensor:
    """3x2 stride-(3,2) mean (ops.rs:1536-1566): six-term sum divided by 6."""
    n, c, h, w = x.shape
    oh, ow = (h - 3) // 3 + 1, (w - 2) // 2 + 1
    x = x[:, :, : oh * 3, : ow * 2].reshape(n, c, oh, 3, ow, 2)
    s = x[:, :, :, 0, :, 0] + x[:, :, :, 0, :, 1] + x[:, :, :, 1, :, 0] + x[:, :, :, 1, :, 1] \
        + x[:, :, :, 2, :, 0] + x[:, :, :, 2, :, 1]
    return s / 6.0


def upsample(x: Tensor, scale: int) -> Tensor:
    if scale == 1:
        return x
    return x.repeat_interleave(scale, dim=2).repeat_interleave(scale, dim=3)


def global_mean(x: Tensor) -> Tensor:
    return x.mean(dim=(2, 3), keepdim=True)


def layer_norm(x: Tensor, weight: np.ndarray, bias: np.ndarray, eps: float = 1e-6) -> Tensor:
    """Two-pass row LayerNorm (kernels/mod.rs:2288-2310)."""
    mean = x.mean(dim=-1, keepdim=True)
    var = ((x - mean) ** 2).mean(dim=-1, keepdim=True)
    inv = 1.0 / torch.sqrt(var + eps)
    return (x - mean) * (inv * t(weight)) + t(bias)


def softmax(x: Tensor) -> Tensor:
    m = x.max(dim=-1, keepdim=True).values
    e = torch.exp(x - m)
    return e * (1.0 / e.sum(dim=-1, keepdim=True))


def linear(x: Tensor, weight: np.ndarray, bias: Optional[np.ndarray]) -> Tensor:
    return F.linear(x, t(weight), None if bias is None else t(bias))


def conv_transpose_2x2(x: Tensor, weight: np.ndarray, bias: np.ndarray) -> Tensor:
    """ConvTranspose 2x2 stride 2, IOHW weight (backend.rs:996-1181)."""
    return F.conv_transpose2d(x, t(weight), t(bias), stride=2)


# ---------------------------------------------------------------------------
# Model assembly (src/cpu/model.rs)
# ---------------------------------------------------------------------------

from importlib import import_module as _imp  # noqa: E402


def _spec():
    return _imp("ppocr_b200.modelspec")


class Conv:
    """A conv with optional folded BN and a fused activation."""

    def __init__(self, weight, bias, stride=(1, 1), pads=(0, 0, 0, 0), groups=1, act=None):
        self.weight, self.bias = weight, bias
        self.stride, self.pads, self.groups, self.act = tuple(stride), tuple(pads), groups, act

    def __call__(self, x: Tensor) -> Tensor:
        y = conv2d(x, self.weight, self.bias, self.stride, self.pads, self.groups)
        return ACTIVATIONS[self.act](y)


def load_conv(w: Weights, prefix: str, cin: int, cout: int, k, stride, pads, bias: bool, groups: int, act=None) -> Conv:
    kh, kw = k
    weight = w.get(f"{prefix}.weight", (cout, cin // groups, kh, kw))
    b = w.get(f"{prefix}.bias", (cout,)) if bias else None
    return Conv(weight, b, stride, pads, groups, act)


def load_conv_bn(w: Weights, prefix: str, cin: int, cout: int, k, stride, pads, bias: bool, groups: int,
                 norm: str = "normalization", act=None) -> Conv:
    kh, kw = k
    weight = w.get(f"{prefix}.convolution.weight", (cout, cin // groups, kh, kw))
    b = w.get(f"{prefix}.convolution.bias", (cout,)) if bias else None
    fw, fb = fold_batch_norm(weight, b, w, f"{prefix}.{norm}", cout)
    return Conv(fw, fb, stride, pads, groups, act)


class SE:
    """Squeeze-excitation: mean -> 1x1 ReLU -> 1x1 -> hard-sigmoid gate."""

    def __init__(self, reduce: Conv, expand: Conv, alpha: float, residual: bool):
        self.reduce, self.expand, self.alpha, self.residual = reduce, expand, alpha, residual

    def gate(self, x: Tensor) -> Tensor:
        pooled = global_mean(x)
        hidden = relu(self.reduce(pooled))
        return hard_sigmoid(self.expand(hidden), self.alpha, 0.5)

    def __call__(self, x: Tensor) -> Tensor:
        g = self.gate(x)
        if self.residual:
            return x + x * g  # residual_mul_in_place (kernels/mod.rs:777-796)
        return x * g


class LcNetBlock:
    """Token depthwise conv -> optional SE -> 1x1 C->2C GELU -> 1x1 2C->C' (+token output)."""

    def __init__(self, w: Weights, prefix: str, blk):
        pad = blk.kernel // 2
        pads = (pad,) * 4
        self.prefix = prefix
        self.residual = blk.residual
        if blk.residual:
            self.token = load_conv(w, f"{prefix}.token_conv", blk.cin, blk.cout, (blk.kernel,) * 2,
                                   blk.stride, pads, True, blk.cin)
        else:
            self.token = load_conv_bn(w, f"{prefix}.token_conv", blk.cin, blk.cin, (blk.kernel,) * 2,
                                      blk.stride, pads, False, blk.cin)
        self.se = None
        if blk.se:
            c = blk.cin
            self.se = SE(load_conv(w, f"{prefix}.token_squeeze_excitation.convolutions.0", c, c // 4, (1, 1), (1, 1), (0,) * 4, True, 1),
                         load_conv(w, f"{prefix}.token_squeeze_excitation.convolutions.2", c // 4, c, (1, 1), (1, 1), (0,) * 4, True, 1),
                         1.0 / 6.0, False)
        self.pw1 = load_conv_bn(w, f"{prefix}.channel_conv1", blk.cin, blk.cin * 2, (1, 1), (1, 1), (0,) * 4, False, 1)
        self.pw2 = load_conv_bn(w, f"{prefix}.channel_conv2", blk.cin * 2, blk.cout, (1, 1), (1, 1), (0,) * 4, False, 1)

    def __call__(self, x: Tensor) -> Tensor:
        y = _trace(f"{self.prefix}.token", self.token(x))
        if self.se is not None:
            y = self.se(y)
        out = self.pw2(gelu(self.pw1(y)))
        # The residual is the token/SE output (backend.rs:504-521, cpu/model.rs:591-602).
        return _trace(f"{self.prefix}.out", y + out if self.residual else out)


class LargeStem:
    def __init__(self, w: Weights, prefix: str, mid: int, out: int):
        c = lambda n, ci, co, k, s, p: load_conv_bn(w, f"{prefix}.{n}", ci, co, k, s, p, False, 1, act="relu")
        self.stem1 = c("stem1", 3, mid, (3, 3), (2, 2), (1, 1, 1, 1))
        self.stem2a = c("stem2a", mid, mid // 2, (2, 2), (1, 1), (0, 0, 1, 1))
        self.stem2b = c("stem2b", mid // 2, mid, (2, 2), (1, 1), (0, 0, 1, 1))
        self.stem3 = c("stem3", mid * 2, mid, (3, 3), (2, 2), (1, 1, 1, 1))
        self.stem4 = c("stem4", mid, out, (1, 1), (1, 1), (0, 0, 0, 0))

    def __call__(self, x: Tensor) -> Tensor:
        e = _trace("stem1", self.stem1(x))
        branch = self.stem2b(self.stem2a(e))
        pooled = max_pool_same_upper(e)
        s3 = _trace("stem3", self.stem3(torch.cat([pooled, branch], dim=1)))
        return _trace("stem4", self.stem4(s3))


class SmallStem:
    def __init__(self, w: Weights, prefix: str, mid: int, out: int):
        self.conv1 = load_conv_bn(w, f"{prefix}.conv1", 3, mid, (3, 3), (2, 2), (1, 1, 1, 1), False, 1, act="gelu")
        self.conv2 = load_conv_bn(w, f"{prefix}.conv2", mid, out, (3, 3), (2, 2), (1, 1, 1, 1), False, 1)

    def __call__(self, x: Tensor) -> Tensor:
        return self.conv2(self.conv1(x))


class Backbone:
    def __init__(self, w: Weights, stages, stem):
        enc = "model.backbone.encoder"
        kind, mid, out = stem
        self.stem = (LargeStem if kind == "large" else SmallStem)(w, f"{enc}.convolution", mid, out)
        self.stages = [[LcNetBlock(w, f"{enc}.blocks.{si}.blocks.{bi}", b) for bi, b in enumerate(st)]
                       for si, st in enumerate(stages)]

    def __call__(self, x: Tensor) -> List[Tensor]:
        h = self.stem(x)
        outs = []
        for stage in self.stages:
            for block in stage:
                h = block(h)
            outs.append(h)
        return outs


def _variant_se(w: Weights, prefix: str, channels: int, reduction: int, residual: bool) -> SE:
    c = channels
    return SE(load_conv(w, f"{prefix}.conv1", c, c // reduction, (1, 1), (1, 1), (0,) * 4, True, 1),
              load_conv(w, f"{prefix}.conv2", c // reduction, c, (1, 1), (1, 1), (0,) * 4, True, 1),
              0.2, residual)


class RepLkFpn:
    """Tiny/small detector neck (cpu/model.rs:1197-1254)."""

    def __init__(self, w: Weights, stage_channels, neck: int, kernel: int):
        self.insert = []
        for i, c in enumerate(stage_channels):
            conv = load_conv(w, f"model.neck.insert_conv.{i}.in_conv", c, neck, (1, 1), (1, 1), (0,) * 4, False, 1)
            se = _variant_se(w, f"model.neck.insert_conv.{i}.squeeze_excitation_block", neck, 4, True)
            self.insert.append((conv, se))
        self.input = []
        pad = kernel // 2
        for i in range(4):
            p = f"model.neck.input_conv.{i}"
            dw = load_conv(w, f"{p}.depthwise_convolution", neck, neck, (kernel, kernel), (1, 1), (pad,) * 4, True, neck)
            pw = load_conv(w, f"{p}.pointwise_convolution", neck, neck // 4, (1, 1), (1, 1), (0,) * 4, False, 1)
            se = _variant_se(w, f"{p}.squeeze_excitation_module", neck // 4, 4, True)
            self.input.append((dw, pw, se))

    def __call__(self, stages: List[Tensor]) -> Tensor:
        fused = [se(conv(f)) for (conv, se), f in zip(self.insert, stages)]
        for i in (2, 1, 0):
            fused[i] = fused[i] + upsample(fused[i + 1], 2)
        feats = [_trace(f"model.neck.input_conv.{i}.out", se(pw(dw(f))))
                 for i, ((dw, pw, se), f) in enumerate(zip(self.input, fused))]
        feats.reverse()
        return torch.cat([upsample(f, s) for f, s in zip(feats, (8, 4, 2, 1))], dim=1)


class RankOne:
    def __init__(self, w: Weights, prefix: str, cin: int, cout: int, k: int):
        weight = w.get(f"{prefix}.weight", (cout, cin, k, k))
        bias = w.get(f"{prefix}.bias", (cout,))
        dw, pw = factor_rank_one(weight, cin, cout, k)
        pad = k // 2
        self.dw = Conv(dw, None, (1, 1), (pad,) * 4, cin)
        self.pw = Conv(pw, bias, (1, 1), (0,) * 4, 1)

    def __call__(self, x: Tensor) -> Tensor:
        return self.pw(self.dw(x))


class Intraclass:
    def __init__(self, w: Weights, prefix: str):
        self.reduce = load_conv(w, f"{prefix}.conv_reduce_channel", 64, 32, (1, 1), (1, 1), (0,) * 4, True, 1)
        self.convs = []
        for ratio, k in (("longratio", 7), ("midratio", 5), ("shortratio", 3)):
            sw = w.get(f"{prefix}.symmetric_conv_long_{ratio}.weight", (32, 32, k, k))
            sb = w.get(f"{prefix}.symmetric_conv_long_{ratio}.bias", (32,))
            vw = w.get(f"{prefix}.vertical_long_to_small_conv_{ratio}.weight", (32, 32, k, 1))
            vb = w.get(f"{prefix}.vertical_long_to_small_conv_{ratio}.bias", (32,))
            hw = w.get(f"{prefix}.horizontal_small_to_long_conv_{ratio}.weight", (32, 32, 1, k))
            hb = w.get(f"{prefix}.horizontal_small_to_long_conv_{ratio}.bias", (32,))
            fw, fb = fuse_intraclass(sw, sb, vw, vb, hw, hb)
            self.convs.append(Conv(fw, fb, (1, 1), (k // 2,) * 4, 1))
        self.final = load_conv_bn(w, f"{prefix}.conv_final", 32, 64, (1, 1), (1, 1), (0,) * 4, True, 1, norm="norm", act="relu")

    def __call__(self, x: Tensor) -> Tensor:
        h = self.reduce(x)
        for conv in self.convs:
            h = conv(h)
        return x + self.final(h)


class MediumNeck:
    """Medium detector neck (cpu/model.rs:948-1067)."""

    def __init__(self, w: Weights):
        self.adjust = [load_conv(w, f"model.neck.input_channel_adjustment_convolution.{i}", c, 256, (1, 1), (1, 1), (0,) * 4, False, 1)
                       for i, c in enumerate((128, 256, 512, 896))]
        self.project = [RankOne(w, f"model.neck.input_feature_projection_convolution.{i}", 256, 64, 9) for i in range(4)]
        self.pan_head = [load_conv(w, f"model.neck.path_aggregation_head_convolution.{i}", 64, 64, (3, 3), (2, 2), (1,) * 4, False, 1)
                         for i in range(3)]
        self.pan_lateral = [RankOne(w, f"model.neck.path_aggregation_lateral_convolution.{i}", 64, 64, 9) for i in range(4)]
        self.intraclass = [Intraclass(w, f"model.neck.intraclass_blocks.{i}") for i in range(4)]

    def __call__(self, stages: List[Tensor]) -> Tensor:
        adjusted = [c(f) for c, f in zip(self.adjust, stages)]
        top_down: List[Tensor] = []
        for f in reversed(adjusted):
            if top_down:
                f = f + upsample(top_down[-1], 2)
            top_down.append(f)
        top_down.reverse()
        projected = [p(f) for p, f in zip(self.project, top_down)]
        bottom_up: List[Tensor] = []
        for i, p in enumerate(projected):
            if bottom_up:
                p = p + self.pan_head[i - 1](bottom_up[-1])
            bottom_up.append(p)
        lateral = [c(f) for c, f in zip(self.pan_lateral, bottom_up)]
        refined = [b(f) for b, f in zip(self.intraclass, lateral)]
        refined.reverse()
        return torch.cat([upsample(f, s) for f, s in zip(refined, (8, 4, 2, 1))], dim=1)


class DetectorHead:
    """3x3 conv BN ReLU -> ConvT 2x2 BN ReLU -> ConvT 2x2 -> sigmoid (cpu/model.rs:1479-1521)."""

    def __init__(self, w: Weights, channels: int):
        hidden = channels // 4
        self.down = load_conv_bn(w, "head.conv_down", channels, hidden, (3, 3), (1, 1), (1,) * 4, False, 1, norm="norm", act="relu")
        uw = w.get("head.conv_up.convolution.weight", (hidden, hidden, 2, 2))
        ub = w.get("head.conv_up.convolution.bias", (hidden,))
        self.up_w, self.up_b = fold_transpose_batch_norm(uw, ub, w, "head.conv_up.norm", hidden)
        self.final_w = w.get("head.conv_final.weight", (hidden, 1, 2, 2))
        self.final_b = w.get("head.conv_final.bias", (1,))

    def logits(self, x: Tensor) -> Tensor:
        h = _trace("head.conv_down", self.down(x))
        h = relu(conv_transpose_2x2(h, self.up_w, self.up_b))
        return conv_transpose_2x2(h, self.final_w, self.final_b)

    def __call__(self, x: Tensor) -> Tensor:
        return sigmoid(self.logits(x))


def validate_input(shape: Sequence[int], detector: bool) -> None:
    """cpu/model.rs:1627-1646."""
    n, c, h, w = shape
    if n <= 0:
        raise ValueError("input batch must not be empty")
    if c != 3:
        raise ValueError("input must have three NCHW channels")
    if h <= 0 or w <= 0:
        raise ValueError("input spatial dimensions must be positive")
    if detector:
        if h % 32 or w % 32:
            raise ValueError("detector input height and width must be multiples of 32")
    else:
        if h != 48:
            raise ValueError("recognizer input height must be 48")
        if w < 5:
            raise ValueError("recognizer input width must be at least 5")


class Detector:
    """cpu::Detector (cpu/model.rs:1537-1625)."""

    def __init__(self, weights: Weights, size: str):
        spec = _spec()
        mid, out = spec.DETECTOR_STEM[size]
        self.size = size
        self.backbone = Backbone(weights, spec.detector_stages(size), ("large", mid, out))
        if size == "medium":
            self.neck = MediumNeck(weights)
        else:
            neck, kernel = spec.DETECTOR_FPN[size]
            self.neck = RepLkFpn(weights, spec.DETECTOR_STAGE_CHANNELS[size], neck, kernel)
        self.head = DetectorHead(weights, spec.DETECTOR_NECK_CHANNELS[size])

    @torch.no_grad()
    def logits(self, x: np.ndarray) -> np.ndarray:
        validate_input(x.shape, True)
        feats = self.backbone(t(x))
        return self.head.logits(self.neck(feats)).numpy()

    @torch.no_grad()
    def forward(self, x: np.ndarray) -> np.ndarray:
        validate_input(x.shape, True)
        feats = self.backbone(t(x))
        return self.head(self.neck(feats)).numpy()


class RecAttention:
    def __init__(self, w: Weights, prefix: str, hidden: int, heads: int):
        self.qkv_w = w.get(f"{prefix}.qkv.weight", (hidden * 3, hidden))
        self.qkv_b = w.get(f"{prefix}.qkv.bias", (hidden * 3,))
        self.proj_w = w.get(f"{prefix}.projection.weight", (hidden, hidden))
        self.proj_b = w.get(f"{prefix}.projection.bias", (hidden,))
        self.hidden, self.heads = hidden, heads

    def __call__(self, x: Tensor) -> Tensor:
        b, s, _ = x.shape
        d = self.hidden // self.heads
        qkv = linear(x, self.qkv_w, self.qkv_b).reshape(b, s, 3, self.heads, d).permute(2, 0, 3, 1, 4)
        q, k, v = qkv[0], qkv[1], qkv[2]
        scores = (q @ k.transpose(2, 3)) * (float(d) ** -0.5)
        out = softmax(scores) @ v
        return linear(out.transpose(1, 2).reshape(b, s, self.hidden), self.proj_w, self.proj_b)


class RecBlock:
    def __init__(self, w: Weights, prefix: str, hidden: int, heads: int, mlp: int):
        self.ln1 = (w.get(f"{prefix}.layer_norm1.weight", (hidden,)), w.get(f"{prefix}.layer_norm1.bias", (hidden,)))
        self.attn = RecAttention(w, f"{prefix}.self_attn", hidden, heads)
        self.ln2 = (w.get(f"{prefix}.layer_norm2.weight", (hidden,)), w.get(f"{prefix}.layer_norm2.bias", (hidden,)))
        self.fc1 = (w.get(f"{prefix}.mlp.fc1.weight", (mlp, hidden)), w.get(f"{prefix}.mlp.fc1.bias", (mlp,)))
        self.fc2 = (w.get(f"{prefix}.mlp.fc2.weight", (hidden, mlp)), w.get(f"{prefix}.mlp.fc2.bias", (hidden,)))

    def __call__(self, x: Tensor) -> Tensor:
        x = x + self.attn(layer_norm(x, *self.ln1))
        h = silu(linear(layer_norm(x, *self.ln2), *self.fc1))
        return x + linear(h, *self.fc2)


class SvtrHead:
    """RecEncoder + classifier of the medium/small recognizer (cpu/model.rs:1775-1875)."""

    def __init__(self, w: Weights, cin: int, hidden: int, mlp: int, classes: int):
        enc = "head.encoder"
        self.skip = load_conv_bn(w, f"{enc}.conv_block.0", cin, hidden, (1, 1), (1, 1), (0,) * 4, False, 1, act="silu")
        self.reduce = load_conv_bn(w, f"{enc}.conv_block.1", cin, hidden, (1, 1), (1, 1), (0,) * 4, False, 1, act="silu")
        self.local = load_conv_bn(w, f"{enc}.conv_block.2", hidden, hidden, (1, 7), (1, 1), (0, 3, 0, 3), False, hidden, act="silu")
        self.blocks = [RecBlock(w, f"{enc}.svtr_block.{i}", hidden, 8, mlp) for i in range(2)]
        self.norm = (w.get(f"{enc}.norm.weight", (hidden,)), w.get(f"{enc}.norm.bias", (hidden,)))
        self.cls = (w.get("head.head.weight", (classes, hidden)), w.get("head.head.bias", (classes,)))

    def logits(self, x: Tensor) -> Tensor:
        residual = self.skip(x)
        h = self.reduce(x)
        h = h + self.local(h)
        n, c, hh, ww = h.shape
        seq = h.flatten(2).transpose(1, 2)
        for blk in self.blocks:
            seq = blk(seq)
        seq = layer_norm(seq, *self.norm)
        h = seq.reshape(n, hh, ww, c).permute(0, 3, 1, 2) + residual
        seq = h.squeeze(2).transpose(1, 2)
        return linear(seq, *self.cls)


class TinyHead:
    """TinyRecognizerHead (cpu/model.rs:1913-1936)."""

    def __init__(self, w: Weights, classes: int):
        c1 = w.get("head.conv1.weight", (160, 1, 5))
        self.c1w, self.c1b = fold_batch_norm(c1, None, w, "head.norm1", 160)
        c2 = w.get("head.conv2.weight", (160, 160, 1))
        self.c2w, self.c2b = fold_batch_norm(c2, None, w, "head.norm2", 160)
        self.fc1 = (w.get("head.fc1.weight", (80, 160)), w.get("head.fc1.bias", (80,)))
        self.fc2 = (w.get("head.fc2.weight", (classes, 80)), w.get("head.fc2.bias", (classes,)))

    def logits(self, x: Tensor) -> Tensor:
        h = hard_swish(conv2d(x, self.c1w.reshape(160, 1, 1, 5), self.c1b, (1, 1), (0, 2, 0, 2), 160))
        h = hard_swish(conv2d(h, self.c2w.reshape(160, 160, 1, 1), self.c2b))
        seq = h.squeeze(2).transpose(1, 2)
        return linear(linear(seq, *self.fc1), *self.fc2)


class Recognizer:
    """cpu::Recognizer (cpu/model.rs:1953-2040).  `logits` is the pre-softmax classifier output."""

    def __init__(self, weights: Weights, size: str):
        spec = _spec()
        self.size = size
        self.backbone = Backbone(weights, spec.recognizer_stages(size), spec.RECOGNIZER_STEM[size])
        classes = spec.RECOGNIZER_CLASSES[size]
        if size == "tiny":
            self.head = TinyHead(weights, classes)
        else:
            cin, hidden, mlp = spec.RECOGNIZER_SVTR[size]
            self.head = SvtrHead(weights, cin, hidden, mlp, classes)

    @torch.no_grad()
    def logits(self, x: np.ndarray) -> np.ndarray:
        validate_input(x.shape, False)
        feat = self.backbone(t(x))[-1]
        return self.head.logits(avg_pool_3x2(feat)).numpy()

    @torch.no_grad()
    def forward(self, x: np.ndarray) -> np.ndarray:
        return softmax(t(self.logits(x))).numpy()


def load_detector(path_or_weights, size: str) -> Detector:
    w = path_or_weights if isinstance(path_or_weights, Weights) else Weights.load(path_or_weights)
    return Detector(w, size)


def load_recognizer(path_or_weights, size: str) -> Recognizer:
    w = path_or_weights if isinstance(path_or_weights, Weights) else Weights.load(path_or_weights)
    return Recognizer(w, size)
