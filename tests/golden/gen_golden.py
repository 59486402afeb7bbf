"""Generates the golden fixtures under tests/golden/ (run once, in a container that has the
reference tree; the outputs are committed and the GPU tests only read them).

  kat_16c_32.npz   the reference's known-answer case: python/01_oracle_and_export.py:51-70
                   restated (seed 0; Conv2d(16 -> 27) makes offset and sigmoid(mask); weight =
                   randn*0.1, bias = 0; x = randn(1,16,32,32); torchvision deform_conv2d).
                   Its output sum is the reference's known answer -30.9894
                   (src/test_dcn.cu:64).
  tv_*.npz         edge cases the reference never tested, with torchvision.ops.deform_conv2d
                   evaluated in float64 as the answer: batch > 1, deformable groups, stride 2,
                   dilation 2, out-of-image offsets, 1x1 and 5x5 kernels, odd sizes.
  npref_*.npz      the reference's own CPU forward (python/dcn_ort_op.py:68-92, imported from the
                   reference tree) on batch > 1 cases with deformable_groups = 1.

Usage:  python tests/golden/gen_golden.py --reference <reference project root>
"""
import argparse
import os
import sys

import numpy as np
import torch
import torch.nn as nn
from torchvision.ops import deform_conv2d

HERE = os.path.dirname(os.path.abspath(__file__))


def kat_fixture():
    N, C, O, K, H, W = 1, 16, 16, 3, 32, 32

    class Block(nn.Module):
        def __init__(self):
            super().__init__()
            self.offset_mask = nn.Conv2d(C, 3 * K * K, K, stride=1, padding=1)
            self.weight = nn.Parameter(torch.randn(O, C, K, K) * 0.1)
            self.bias = nn.Parameter(torch.zeros(O))

    torch.manual_seed(0)
    blk = Block().eval()
    x = torch.randn(N, C, H, W)
    with torch.no_grad():
        om = blk.offset_mask(x)
        off, msk = om[:, :2 * K * K], torch.sigmoid(om[:, 2 * K * K:])
        y = deform_conv2d(x, off, blk.weight, blk.bias, stride=(1, 1), padding=(1, 1),
                          dilation=(1, 1), mask=msk)
    return dict(x=x.numpy(), offset=off.numpy(), mask=msk.numpy(),
                weight=blk.weight.detach().numpy(), bias=blk.bias.detach().numpy(), y=y.numpy(),
                stride=1, padding=1, dilation=1, groups=1)


EDGE_CASES = {
    # name: (N, C, O, H, W, K, stride, pad, dil, dg, offset_std, outlier_frac, seed)
    "tv_n2_dg2_s2": (2, 16, 24, 11, 13, 3, 2, 1, 1, 2, 1.5, 0.05, 1),
    "tv_d2_p2_dg8": (1, 64, 32, 12, 12, 3, 1, 2, 2, 8, 2.0, 0.0, 2),
    "tv_oob": (1, 8, 8, 9, 9, 3, 1, 1, 1, 1, 0.5, 0.3, 3),
    "tv_k1": (2, 32, 16, 7, 9, 1, 1, 0, 1, 1, 0.7, 0.0, 4),
    "tv_k5": (1, 16, 16, 10, 10, 5, 1, 2, 1, 1, 0.7, 0.0, 5),
    "tv_odd": (3, 24, 40, 7, 5, 3, 1, 1, 1, 3, 1.0, 0.1, 6),
}


def edge_fixture(N, C, O, H, W, K, s, p, d, dg, ostd, outl, seed):
    g = torch.Generator().manual_seed(seed)
    Ho = (H + 2 * p - d * (K - 1) - 1) // s + 1
    Wo = (W + 2 * p - d * (K - 1) - 1) // s + 1
    x = torch.randn(N, C, H, W, generator=g)
    w = (torch.rand(O, C, K, K, generator=g) * 2 - 1) / np.sqrt(C * K * K)
    b = (torch.rand(O, generator=g) * 2 - 1) * 0.05
    off = torch.randn(N, 2 * dg * K * K, Ho, Wo, generator=g) * ostd
    if outl > 0:
        sel = torch.rand(off.shape, generator=g) < outl
        off = torch.where(sel, torch.sign(torch.randn(off.shape, generator=g)) * 70.0, off)
    msk = torch.sigmoid(torch.randn(N, dg * K * K, Ho, Wo, generator=g))
    y = deform_conv2d(x.double(), off.double(), w.double(), b.double(), stride=(s, s),
                      padding=(p, p), dilation=(d, d), mask=msk.double())
    return dict(x=x.numpy(), offset=off.numpy(), mask=msk.numpy(), weight=w.numpy(),
                bias=b.numpy(), y=y.numpy(), stride=s, padding=p, dilation=d, groups=dg)


NPREF_CASES = {
    "npref_n3": (3, 16, 8, 10, 12, 3, 1, 1, 1, 1, 0.8, 0.05, 11),
    "npref_n2_s2_d2": (2, 8, 8, 13, 11, 3, 2, 2, 2, 1, 1.2, 0.0, 12),
}


def npref_fixture(ref_python_dir, N, C, O, H, W, K, s, p, d, dg, ostd, outl, seed):
    sys.path.insert(0, ref_python_dir)
    try:
        import dcn_ort_op  # the reference's numpy im2col + GEMM forward
    finally:
        sys.path.pop(0)
    fx = edge_fixture(N, C, O, H, W, K, s, p, d, dg, ostd, outl, seed)
    fx["y"] = dcn_ort_op.dcn_v2_forward(fx["x"], fx["offset"], fx["mask"], fx["weight"],
                                        fx["bias"], stride=s, pad=p, dil=d)
    return fx


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the reference project (holds python/dcn_ort_op.py)")
    args = ap.parse_args()
    kat = kat_fixture()
    print("kat y.sum =", float(kat["y"].sum()))
    np.savez_compressed(os.path.join(HERE, "kat_16c_32.npz"), **kat)
    for name, cfg in EDGE_CASES.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **edge_fixture(*cfg))
    ref_py = os.path.join(args.reference, "python")
    if os.path.isdir(ref_py):
        for name, cfg in NPREF_CASES.items():
            np.savez_compressed(os.path.join(HERE, name + ".npz"), **npref_fixture(ref_py, *cfg))
    else:
        print("reference tree not found; npref fixtures not regenerated")


if __name__ == "__main__":
    main()
