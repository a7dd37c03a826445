"""The algebra of the tap-shifted convolution (newch_b200/csrc/k_convtap.cu), in numpy on CPU.

x [N][C][H][W] is packed into a position-major matrix over the zero-padded grid, row
v = n*Hp*Wp + h'*Wp + w' (Hp = H + 2ph, Wp = W + 2pw), channels padded to a multiple of 32; output
pixel (oh, ow) sits at the same row, and filter tap (ki, kj) is the row shift s = ki*dh*Wp + kj*dw:
    forward  Y~[v]    = sum_tap X~[v + s] Wf[tap]^T
    dX       dX~[u]   = sum_tap G~[u - s] Wx[tap]^T       (G~ = dY packed on the same grid, zero rows
                                                           where (oh, ow) is outside the output)
    dW[tap]           = sum_v X~[v + s]^T G~[v]
with rows past either end of a packed matrix reading zero (the TMA's fill). This test restates those
three GEMMs with numpy row shifts and checks them against the oracle's convolution and its gradients
(the reference's ops_conv.c semantics) over the padding, dilation and kernel shapes the GPU tests use."""

from __future__ import annotations

import numpy as np
import pytest

import ncoracle as O


def _pack(src, Hp, Wp, eh, ew, Kp):
    N, C, Hs, Ws = src.shape
    out = np.zeros((N, Hp, Wp, Kp))
    out[:, eh:eh + Hs, ew:ew + Ws, :C] = src.transpose(0, 2, 3, 1)
    return out.reshape(N * Hp * Wp, Kp)


def _shifted(M, s):
    """rows M[v + s], zero outside the matrix"""
    out = np.zeros_like(M)
    n = len(M)
    lo, hi = max(0, -s), min(n, n - s)
    if hi > lo:
        out[lo:hi] = M[lo + s:hi + s]
    return out


@pytest.mark.parametrize("xs,wk,pad,dil", [
    ((3, 4, 9, 11), (5, 3, 3), (1, 1), (1, 1)),
    ((2, 12, 12, 12), (24, 5, 5), (2, 2), (1, 1)),
    ((2, 8, 15, 15), (20, 3, 3), (2, 2), (2, 2)),
    ((4, 40, 6, 5), (33, 1, 3), (0, 1), (1, 1)),
    ((5, 20, 10, 9), (12, 3, 2), (0, 1), (1, 1)),
    ((2, 40, 7, 7), (7, 3, 3), (0, 0), (1, 1)),
])
def test_tap_shift_gemms_equal_convolution(xs, wk, pad, dil):
    rng = np.random.default_rng(0)
    (N, C, H, W), (OC, KH, KW), (ph, pw), (dh, dw) = xs, wk, pad, dil
    X = rng.standard_normal(xs).astype(np.float32)
    Wt = rng.standard_normal((OC, C, KH, KW)).astype(np.float32)
    Hp, Wp = H + 2 * ph, W + 2 * pw
    OH, OW = Hp - dh * (KH - 1), Wp - dw * (KW - 1)
    Cp, OCp, T = -(-C // 32) * 32, -(-OC // 32) * 32, KH * KW
    shifts = [ki * dh * Wp + kj * dw for ki in range(KH) for kj in range(KW)]

    Xp = _pack(X.astype(np.float64), Hp, Wp, ph, pw, Cp)
    Wf = np.zeros((OC, T, Cp))
    Wf[:, :, :C] = Wt.reshape(OC, C, T).transpose(0, 2, 1)
    D = sum(_shifted(Xp, shifts[t]) @ Wf[:, t, :].T for t in range(T))
    Y = D.reshape(N, Hp, Wp, OC)[:, :OH, :OW].transpose(0, 3, 1, 2)
    Y_ref = O.conv2d(X, Wt, None, stride=(1, 1), pad=pad, dil=dil)
    assert np.abs(Y - Y_ref).max() <= 1e-5 * np.abs(Y_ref).max()

    G = rng.standard_normal(Y_ref.shape).astype(np.float32)
    Gp = _pack(G.astype(np.float64), Hp, Wp, 0, 0, OCp)
    Wx = np.zeros((C, T, OCp))
    Wx[:, :, :OC] = Wt.reshape(OC, C, T).transpose(1, 2, 0)
    DX = sum(_shifted(Gp, -shifts[t]) @ Wx[:, t, :].T for t in range(T))
    dX = DX.reshape(N, Hp, Wp, C)[:, ph:ph + H, pw:pw + W].transpose(0, 3, 1, 2)
    DW = np.stack([_shifted(Xp, shifts[t]).T @ Gp for t in range(T)])  # [T][Cp][OCp]
    dW = DW[:, :C, :OC].transpose(2, 1, 0).reshape(OC, C, KH, KW)
    dx_ref, dw_ref, _ = O.conv2d_grads(X, Wt, G, stride=(1, 1), pad=pad, dil=dil)
    assert np.abs(dX - dx_ref).max() <= 1e-5 * np.abs(dx_ref).max()
    assert np.abs(dW - dw_ref).max() <= 1e-5 * np.abs(dw_ref).max()
