"""Seeded synthetic inputs for the DCNv2 layer workloads measured and tested here.

No dataset is involved: every workload is a single deformable-convolution layer whose inputs are
drawn from fixed distributions with torch.Generator on the CPU (bit-reproducible), then moved to
the target device. The shapes and distributions are:

  fp32_n1_256c_64     N=1,  C=O=256, 64x64, K3 s1 p1 d1 dg1, fp32. x~N(0,1); W kaiming-uniform
                      (a=sqrt(5)); b~U(-0.05,0.05); offset~N(0,0.5^2) with ~5% of entries set to
                      +-70 (out-of-image samples); mask=sigmoid(N(0,1)).
  fp16_n64_256c_64    N=64, same layer in fp16, identity-like offset~N(0,0.1^2),
                      mask=sigmoid(N(3,0.5^2)).
  int8_n64_256c_64    N=64, x and W quantised per tensor (scale=max|v|/127, round half away from
                      zero, clamp +-127); offset/mask fp32 drawn as in fp32_n1_256c_64.
  fpn_fp16_b32        B=32, 256 channels, levels 64,32,16,8,4 (one layer each), fp16 with the
                      fp16_n64_256c_64 offset/mask distributions.
  big_512c_128_dg8    C=O=512, 128x128, K3 d2 p2 dg8, offset~N(0,2^2), mask=sigmoid(N(0,1));
                      x and W as in fp32_n1_256c_64; fp16 or int8.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, Optional

import torch


@dataclass
class Layer:
    n: int
    c: int
    h: int
    w: int
    out_c: int
    kernel: int = 3
    stride: int = 1
    padding: int = 1
    dilation: int = 1
    groups: int = 1

    @property
    def ho(self) -> int:
        return (self.h + 2 * self.padding - self.dilation * (self.kernel - 1) - 1) // self.stride + 1

    @property
    def wo(self) -> int:
        return (self.w + 2 * self.padding - self.dilation * (self.kernel - 1) - 1) // self.stride + 1

    @property
    def flops(self) -> int:
        """2 * N * O * C * K^2 * Ho * Wo (multiply-adds x 2; sampling arithmetic excluded)."""
        return 2 * self.n * self.out_c * self.c * self.kernel ** 2 * self.ho * self.wo


@dataclass
class Inputs:
    layer: Layer
    precision: str            # "fp32" | "fp16" | "int8"
    x: torch.Tensor
    offset: torch.Tensor
    mask: torch.Tensor
    weight: torch.Tensor
    bias: torch.Tensor
    x_scale: float = 1.0
    w_scale: float = 1.0
    # fp32 originals of quantised / half tensors (for reference comparisons)
    extra: Dict[str, torch.Tensor] = field(default_factory=dict)

    def to(self, device) -> "Inputs":
        mv = lambda t: t.to(device).contiguous()
        return Inputs(self.layer, self.precision, mv(self.x), mv(self.offset), mv(self.mask),
                      mv(self.weight), mv(self.bias), self.x_scale, self.w_scale,
                      {k: v for k, v in self.extra.items()})

    def tensors(self):
        return self.x, self.offset, self.mask, self.weight, self.bias

    def images(self, start: int, stop: int) -> "Inputs":
        """Images [start, stop) of the batch (x, offset, mask sliced; weight, bias shared)."""
        L = self.layer
        sub = Layer(stop - start, L.c, L.h, L.w, L.out_c, L.kernel, L.stride, L.padding,
                    L.dilation, L.groups)
        cut = lambda t: t[start:stop].contiguous()
        return Inputs(sub, self.precision, cut(self.x), cut(self.offset), cut(self.mask),
                      self.weight, self.bias, self.x_scale, self.w_scale,
                      {k: (cut(v) if k == "x_f32" else v) for k, v in self.extra.items()})

    @property
    def input_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors())

    @property
    def output_bytes(self) -> int:
        esz = 2 if self.precision == "fp16" else 4
        L = self.layer
        return L.n * L.out_c * L.ho * L.wo * esz


def quantize_sym(v: torch.Tensor):
    """Per-tensor symmetric int8 quantiser of the reference INT8 tests
    (src/test_dcn_int8.cu:31-42): scale = max|v|/127 (1 if all zero),
    q = clamp(lroundf(v/scale), -127, 127) with round-half-away-from-zero."""
    v = v.float()
    mx = float(v.abs().max()) if v.numel() else 0.0
    scale = torch.tensor(mx, dtype=torch.float32) / torch.tensor(127.0, dtype=torch.float32)
    scale = float(scale) if mx > 0 else 1.0
    r = v / torch.tensor(scale, dtype=torch.float32)
    q = torch.sign(r) * torch.floor(r.abs() + 0.5)
    q = q.clamp_(-127, 127).to(torch.int8)
    return q, scale


def _kaiming_uniform(o, c, k, g):
    fan_in = c * k * k
    bound = 1.0 / math.sqrt(fan_in)  # kaiming_uniform_(a=sqrt(5)) bound = sqrt(6/((1+5)*fan_in))
    return (torch.rand((o, c, k, k), generator=g) * 2 - 1) * bound


def make_layer_inputs(layer: Layer, precision: str, offset_std: float, mask_mean: float,
                      mask_std: float, outlier_frac: float = 0.0, outlier_mag: float = 70.0,
                      seed: int = 0) -> Inputs:
    g = torch.Generator().manual_seed(seed)
    L = layer
    T = L.kernel * L.kernel
    x = torch.randn((L.n, L.c, L.h, L.w), generator=g)
    w = _kaiming_uniform(L.out_c, L.c, L.kernel, g)
    b = (torch.rand((L.out_c,), generator=g) * 2 - 1) * 0.05
    off = torch.randn((L.n, 2 * L.groups * T, L.ho, L.wo), generator=g) * offset_std
    if outlier_frac > 0:
        sel = torch.rand(off.shape, generator=g) < outlier_frac
        sgn = torch.where(torch.rand(off.shape, generator=g) < 0.5, -1.0, 1.0)
        off = torch.where(sel, sgn * outlier_mag, off)
    msk = torch.sigmoid(torch.randn((L.n, L.groups * T, L.ho, L.wo), generator=g) * mask_std
                        + mask_mean)
    extra = {"x_f32": x, "w_f32": w}
    if precision == "fp32":
        return Inputs(L, precision, x, off, msk, w, b, extra=extra)
    if precision == "fp16":
        return Inputs(L, precision, x.half(), off.half(), msk.half(), w.half(), b.half(),
                      extra=extra)
    if precision == "int8":
        xq, xs = quantize_sym(x)
        wq, ws = quantize_sym(w)
        return Inputs(L, precision, xq, off, msk, wq, b, xs, ws, extra=extra)
    raise ValueError(precision)


WORKLOADS = ("fp32_n1_256c_64", "fp16_n64_256c_64", "int8_n64_256c_64", "fpn_fp16_b32",
             "big_512c_128_dg8", "big_512c_128_dg8_int8")


def workload(name: str, n: Optional[int] = None, precision: Optional[str] = None,
             level: Optional[int] = None, seed: int = 0) -> Inputs:
    """Builds one workload (n overrides the batch; level selects an FPN level size)."""
    if name == "fp32_n1_256c_64":
        return make_layer_inputs(Layer(n or 1, 256, 64, 64, 256), "fp32", 0.5, 0.0, 1.0,
                                 outlier_frac=0.05, seed=seed)
    if name == "fp16_n64_256c_64":
        return make_layer_inputs(Layer(n or 64, 256, 64, 64, 256), "fp16", 0.1, 3.0, 0.5,
                                 seed=seed)
    if name == "int8_n64_256c_64":
        return make_layer_inputs(Layer(n or 64, 256, 64, 64, 256), "int8", 0.5, 0.0, 1.0,
                                 outlier_frac=0.05, seed=seed)
    if name == "fpn_fp16_b32":
        s = level or 64
        return make_layer_inputs(Layer(n or 32, 256, s, s, 256), "fp16", 0.1, 3.0, 0.5,
                                 seed=seed + s)
    if name in ("big_512c_128_dg8", "big_512c_128_dg8_int8"):
        prec = precision or ("int8" if name.endswith("int8") else "fp16")
        return make_layer_inputs(Layer(n or 16, 512, 128, 128, 512, 3, 1, 2, 2, 8),
                                 prec, 2.0, 0.0, 1.0, seed=seed)
    raise KeyError(name)


FPN_LEVELS = (64, 32, 16, 8, 4)


def workload_parts(name: str, n: Optional[int] = None, seed: int = 0):
    """The layers one step of a workload runs: the five FPN levels (P3..P7) of fpn_fp16_b32, a
    single layer otherwise."""
    if name == "fpn_fp16_b32":
        return [workload(name, n=n, level=s, seed=seed) for s in FPN_LEVELS]
    return [workload(name, n=n, seed=seed)]


def head_inputs(layer: Layer, offset_std: float = 0.1, mask_logit: float = 3.0, seed: int = 0):
    """Weights of an offset / mask head Conv2d(C -> 3*dg*K*K, K, padding (K-1)/2) for `layer`,
    drawn so that on x ~ N(0, 1) the offsets come out ~N(0, offset_std^2) and the mask logits
    ~N(mask_logit, offset_std^2) (the fp16 workload's identity-like distributions): weight
    uniform with that standard deviation over the fan-in, bias 0 for the offsets and mask_logit
    for the mask. Returned as fp32 CPU tensors ([3*dg*K*K, C, K, K], [3*dg*K*K])."""
    g = torch.Generator().manual_seed(seed + 7919)
    L = layer
    n_head = 3 * L.groups * L.kernel ** 2
    fan_in = L.c * L.kernel ** 2
    bound = offset_std * math.sqrt(3.0 / fan_in)  # uniform(-b, b) has std b / sqrt(3)
    w = (torch.rand((n_head, L.c, L.kernel, L.kernel), generator=g) * 2 - 1) * bound
    b = torch.zeros(n_head)
    b[2 * L.groups * L.kernel ** 2:] = mask_logit
    return w, b
