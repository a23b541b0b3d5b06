"""CPU oracle for the NOVA F(6,3) Winograd 3x3 stride-1 convolution forward.

TEST INFRASTRUCTURE ONLY.  This module is the checker for the CUDA library in
``nova-wino-amd_b200/``; it is imported by ``tests/``, by
``__graft_entry__.smoke()`` and by the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py``.  The product path never imports it, and there is no CPU
fallback anywhere in the library.

It restates, in numpy float32, the algorithm of the reference implementation
(Jayluci4/nova-wino-amd, HIP + rocBLAS for MI300X):

* transform matrices            ``csrc/nova_winograd.hip:68-97`` (points
                                {0, +-3/5, +-1, +-7/6, inf}, ``:45``)
* their FP16 upload             ``csrc/nova_winograd.hip:103-131`` (A and B are
                                stored as ``__half``; G stays FP32)
* tiling                        ``csrc/nova_winograd.hip:617-631``
* filter transform              ``csrc/nova_winograd.hip:214-255`` (U = G w G^T
                                in FP32, stored FP16 as ``U[pos][c][k]``)
* input transform               ``csrc/nova_winograd.hip:338-392`` (V = B^T d B
                                with fused zero padding, tile origin
                                ``th*6-pad``, stored FP16 as ``V[pos][bp][c]``)
* batched GEMM                  rocBLAS ``gemm_strided_batched_ex`` at
                                ``csrc/nova_winograd.hip:534-548`` (64 GEMMs,
                                FP16 in, FP32 accumulate, FP16 out ``M[pos][bp][k]``)
* output transform              ``csrc/nova_winograd.hip:398-450`` (Y = A M A^T,
                                bounds-checked NCHW store, FP16)

Two modes:

``"ref"``   FP32 arithmetic with the reference's storage roundings: FP16 A/B
            constants, FP16 V, U, M and output.  This is the reference's
            numerics; the CUDA path is compared against it.
``"exact"`` FP32 everywhere, FP32 constants, no intermediate rounding.  The
            error of "ref" against an FP64 direct convolution is the accuracy
            bar (the CUDA path must be no worse than 1.1x of it).

The GEMM arithmetic of the reference lives in rocBLAS (ROCm 6.3, not vendored);
its published contract -- D = alpha*A*B + beta*C with FP32 compute and FP16
result rounding to nearest -- is what ``gemm`` restates.
"""

from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------------------
# a1: NOVA transform matrices, csrc/nova_winograd.hip:68-97 (host tables).
# ---------------------------------------------------------------------------

NOVA_POINTS = (0.0, 3.0 / 5.0, -3.0 / 5.0, 1.0, -1.0, 7.0 / 6.0, -7.0 / 6.0)  # + infinity

A_TABLE = np.array([
    [1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 0.0000000000],
    [0.0000000000, 0.6000000000, -0.6000000000, 1.0000000000, -1.0000000000, 1.1666666667, -1.1666666667, 0.0000000000],
    [0.0000000000, 0.3600000000, 0.3600000000, 1.0000000000, 1.0000000000, 1.3611111111, 1.3611111111, 0.0000000000],
    [0.0000000000, 0.2160000000, -0.2160000000, 1.0000000000, -1.0000000000, 1.5879629630, -1.5879629630, 0.0000000000],
    [0.0000000000, 0.1296000000, 0.1296000000, 1.0000000000, 1.0000000000, 1.8526234568, 1.8526234568, 0.0000000000],
    [0.0000000000, 0.0777600000, -0.0777600000, 1.0000000000, -1.0000000000, 2.1613940329, -2.1613940329, 1.0000000000],
])

B_TABLE = np.array([
    [-0.4900000000, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
    [0.0, 0.8166666667, -0.8166666667, 0.4900000000, -0.4900000000, 0.4200000000, -0.4200000000, -0.4900000000],
    [2.2111111111, 1.3611111111, 1.3611111111, 0.4900000000, 0.4900000000, 0.3600000000, 0.3600000000, 0.0],
    [0.0, -1.4166666667, 1.4166666667, -1.7211111111, 1.7211111111, -1.5866666667, 1.5866666667, 2.2111111111],
    [-2.7211111111, -2.3611111111, -2.3611111111, -1.7211111111, -1.7211111111, -1.3600000000, -1.3600000000, 0.0],
    [0.0, 0.6000000000, -0.6000000000, 1.0000000000, -1.0000000000, 1.1666666667, -1.1666666667, -2.7211111111],
    [1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 1.0000000000, 0.0],
    [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0000000000],
])

G_TABLE = np.array([
    [-2.0408163265, 0.0000000000, 0.0000000000],
    [2.1677302997, 1.3006381798, 0.7803829079],
    [2.1677302997, -1.3006381798, 0.7803829079],
    [-2.1634615385, -2.1634615385, -2.1634615385],
    [-2.1634615385, 2.1634615385, -2.1634615385],
    [1.0161394021, 1.1854959691, 1.3830786306],
    [1.0161394021, -1.1854959691, 1.3830786306],
    [0.0000000000, 0.0000000000, 1.0000000000],
])

M_OUT, R_FILT, N_TILE = 6, 3, 8


def matrices(mode: str = "ref"):
    """Return (A, B, G) as float32 in the precision the given mode computes with.

    "ref": A and B go through float -> __half exactly as
    ``upload_transform_matrices`` does (csrc/nova_winograd.hip:103-131); G stays FP32.
    """
    A = A_TABLE.astype(np.float32)
    B = B_TABLE.astype(np.float32)
    G = G_TABLE.astype(np.float32)
    if mode == "ref":
        A = A.astype(np.float16).astype(np.float32)
        B = B.astype(np.float16).astype(np.float32)
    elif mode != "exact":
        raise ValueError(f"unknown oracle mode {mode!r}")
    return A, B, G


def cook_toom_residual() -> float:
    """Max |error| of the 1-D F(6,3) identity  y = A [(G g) * (B^T d)]  in FP64.

    Checks the reference tables against the definition of a Winograd minimal
    filter: for any 8-sample signal d and 3-tap filter g the 6 outputs equal
    the valid correlation.
    """
    rng = np.random.default_rng(0)
    worst = 0.0
    for _ in range(64):
        d = rng.standard_normal(8)
        g = rng.standard_normal(3)
        y = A_TABLE @ ((G_TABLE @ g) * (B_TABLE.T @ d))
        ref = np.array([d[i:i + 3] @ g for i in range(6)])
        worst = max(worst, float(np.max(np.abs(y - ref))))
    return worst


# ---------------------------------------------------------------------------
# a2: tiling, csrc/nova_winograd.hip:617-631 (also ops.py:128-144).
# ---------------------------------------------------------------------------

def compute_tiling(H: int, W: int, pad: int):
    """(nh, nw, H_out, W_out) exactly as the reference computes them."""
    m, n = M_OUT, N_TILE
    H_out = H + 2 * pad - 2
    W_out = W + 2 * pad - 2
    H_pad = H_out + n - 1
    W_pad = W_out + n - 1
    H_pad += (m - (H_pad - n) % m) % m
    W_pad += (m - (W_pad - n) % m) % m
    return (H_pad - n) // m + 1, (W_pad - n) // m + 1, H_out, W_out


def live_tiling(H: int, W: int, pad: int):
    """(nh, nw): tiles that cover at least one output pixel, ceil(H_out/6)."""
    H_out = H + 2 * pad - 2
    W_out = W + 2 * pad - 2
    return -(-H_out // M_OUT), -(-W_out // M_OUT)


# ---------------------------------------------------------------------------
# a3-a6: the three passes.
# ---------------------------------------------------------------------------

def _round(x: np.ndarray, mode: str) -> np.ndarray:
    return x.astype(np.float16) if mode == "ref" else x.astype(np.float32)


def filter_transform(w: np.ndarray, mode: str = "ref") -> np.ndarray:
    """U in the reference GEMM layout [64][C][K] (k fastest).

    csrc/nova_winograd.hip:214-255: U[pos][k][c] = (G w_kc G^T)[pos] in FP32,
    written at ``pos*K*C + k + c*K`` and rounded to FP16.
    """
    _, _, G = matrices(mode)
    K, C = w.shape[:2]
    u = G @ w.astype(np.float32) @ G.T                       # [K, C, 8, 8]
    u = u.transpose(2, 3, 1, 0).reshape(64, C, K)
    return _round(np.ascontiguousarray(u), mode)


def input_tiles(x: np.ndarray, nh: int, nw: int, pad: int) -> np.ndarray:
    """Overlapping 8x8 windows at stride 6, origin (th*6-pad, tw*6-pad), zero padded.

    Returns float32 [B, C, nh, nw, 8, 8]; csrc/nova_winograd.hip:358-370.
    """
    Bn, C, H, W = x.shape
    Hp = (nh - 1) * 6 + 8
    Wp = (nw - 1) * 6 + 8
    xp = np.zeros((Bn, C, Hp, Wp), dtype=np.float32)
    hs, ws = min(H, Hp - pad), min(W, Wp - pad)
    xp[:, :, pad:pad + hs, pad:pad + ws] = x[:, :, :hs, :ws].astype(np.float32)
    win = np.lib.stride_tricks.sliding_window_view(xp, (8, 8), axis=(2, 3))
    return np.ascontiguousarray(win[:, :, ::6, ::6])


def input_transform(x: np.ndarray, nh: int, nw: int, pad: int, mode: str = "ref") -> np.ndarray:
    """V in the reference GEMM layout [64][B*P][C] (c fastest).

    csrc/nova_winograd.hip:372-391: temp = B^T d, V = temp B, stored at
    ``pos*C*BP + c + bp*C`` with bp = b*P + th*nw + tw.
    """
    _, Bm, _ = matrices(mode)
    Bn, C = x.shape[:2]
    d = input_tiles(x, nh, nw, pad)
    v = Bm.T @ d @ Bm                                        # [B, C, nh, nw, 8, 8]
    v = v.transpose(4, 5, 0, 2, 3, 1).reshape(64, Bn * nh * nw, C)
    return _round(np.ascontiguousarray(v), mode)


def gemm(U: np.ndarray, V: np.ndarray, mode: str = "ref") -> np.ndarray:
    """M[pos][bp][k] = sum_c V[pos][bp][c] * U[pos][c][k], FP32 accumulate.

    rocBLAS gemm_strided_batched_ex at csrc/nova_winograd.hip:534-548 (column
    major M(KxBP) = U(KxC) V(CxBP), which is this row-major product).
    """
    m = np.matmul(V.astype(np.float32), U.astype(np.float32))
    return _round(m, mode)


def output_transform(M: np.ndarray, Bn: int, nh: int, nw: int, H_out: int, W_out: int,
                     mode: str = "ref") -> np.ndarray:
    """y NCHW [B, K, H_out, W_out] from M[64][B*P][K]; csrc/nova_winograd.hip:420-449."""
    A, _, _ = matrices(mode)
    K = M.shape[2]
    m = M.astype(np.float32).reshape(8, 8, Bn, nh, nw, K).transpose(2, 5, 3, 4, 0, 1)
    y = A @ m @ A.T                                          # [B, K, nh, nw, 6, 6]
    y = _round(y, mode)
    y = y.transpose(0, 1, 2, 4, 3, 5).reshape(Bn, K, nh * 6, nw * 6)
    return np.ascontiguousarray(y[:, :, :H_out, :W_out])


def nova_forward(x: np.ndarray, w: np.ndarray, pad: int = 1, mode: str = "ref",
                 live_tiles_only: bool = True) -> np.ndarray:
    """Whole NOVA forward on CPU.  ``x`` [B,C,H,W] (FP16 values), ``w`` [K,C,3,3] FP32.

    Tiles beyond ceil(H_out/6) (the reference's over-tiling) lie entirely in the
    padding and write nothing (csrc/nova_winograd.hip:446), so skipping them
    changes no output value.
    """
    Bn, C, H, W = x.shape
    nh, nw, H_out, W_out = compute_tiling(H, W, pad)
    if live_tiles_only:
        nh, nw = live_tiling(H, W, pad)
    U = filter_transform(w, mode)
    V = input_transform(x, nh, nw, pad, mode)
    M = gemm(U, V, mode)
    return output_transform(M, Bn, nh, nw, H_out, W_out, mode)


# ---------------------------------------------------------------------------
# The same three passes in the reference kernels' exact operation order.
#
# Each reference kernel accumulates its 8 (or 3x3) products one after another
# in FP32, and the compiler contracts ``acc += a * b`` into a fused
# multiply-add.  These restatements do the same, emulating each FMA in FP64
# (the product of two FP32 numbers is exact there; the sum is then rounded to
# FP32 -- a double rounding that differs from a true FMA with probability of
# order 2^-29 per operation).  Their outputs match the reference kernels bit
# for bit; the fast "ref" functions above differ from them only by FP32
# summation order.
# ---------------------------------------------------------------------------

def _fma(acc, a, b):
    """fl32(acc + a*b) with a single product rounding (FMA), elementwise."""
    return (acc.astype(np.float64) + a.astype(np.float64) * b.astype(np.float64)).astype(np.float32)


def filter_transform_seq(w: np.ndarray) -> np.ndarray:
    """U[64][C][K] FP16 as filter_transform_kernel computes it
    (csrc/nova_winograd.hip:243-254): for (p, q) in order,
    result = fma(fl32(G[row][p] * w[p][q]), G^T[q][col], result)."""
    _, _, G = matrices("ref")
    K, C = w.shape[:2]
    w = w.astype(np.float32)
    acc = np.zeros((8, 8, K, C), dtype=np.float32)
    for p in range(3):
        for q in range(3):
            t = (G[:, p][:, None, None] * w[None, :, :, p, q]).astype(np.float32)  # [row, K, C]
            acc = _fma(acc, t[:, None], G[:, q][None, :, None, None])
    return np.ascontiguousarray(acc.reshape(64, K, C).transpose(0, 2, 1)).astype(np.float16)


def input_transform_seq(x: np.ndarray, nh: int, nw: int, pad: int) -> np.ndarray:
    """V[64][B*P][C] FP16 as input_transform_kernel (csrc/nova_winograd.hip:181-199)
    and input_transform_kernel_mt (:372-387) compute it:
    temp[r][c] = sum_k fma(B^T[r][k], d[k][c]) in k order, then
    V[r][c] = sum_k fma(temp[r][k], B[k][c]) in k order."""
    _, Bm, _ = matrices("ref")
    Bn, C = x.shape[:2]
    d = input_tiles(x, nh, nw, pad)                       # [..., 8 (k), 8 (c)]
    temp = np.zeros(d.shape, dtype=np.float32)
    for k in range(8):
        temp = _fma(temp, Bm[k, :][:, None], d[..., k:k + 1, :])      # B^T[r][k] = B[k][r]
    v = np.zeros(d.shape, dtype=np.float32)
    for k in range(8):
        v = _fma(v, temp[..., :, k:k + 1], Bm[k, :][None, :])
    v = v.transpose(4, 5, 0, 2, 3, 1).reshape(64, Bn * nh * nw, C)
    return np.ascontiguousarray(v).astype(np.float16)


def output_transform_seq(M: np.ndarray, Bn: int, nh: int, nw: int, H_out: int,
                         W_out: int) -> np.ndarray:
    """y FP16 NCHW as output_transform_kernel (csrc/nova_winograd.hip:305-327)
    and output_transform_kernel_mt (:426-448) compute it:
    temp[r][c] = sum_p fma(A[r][p], m[p][c]), y[r][c] = sum_p fma(temp[r][p], A^T[p][c])."""
    A, _, _ = matrices("ref")
    K = M.shape[2]
    m = M.astype(np.float32).reshape(8, 8, Bn, nh, nw, K).transpose(2, 5, 3, 4, 0, 1)
    temp = np.zeros(m.shape[:-2] + (6, 8), dtype=np.float32)
    for p in range(8):
        temp = _fma(temp, A[:, p][:, None], m[..., p:p + 1, :])
    y = np.zeros(m.shape[:-2] + (6, 6), dtype=np.float32)
    for p in range(8):
        y = _fma(y, temp[..., :, p:p + 1], A[:, p][None, :])
    y = y.astype(np.float16).transpose(0, 1, 2, 4, 3, 5).reshape(Bn, K, nh * 6, nw * 6)
    return np.ascontiguousarray(y[:, :, :H_out, :W_out])


def gemm_scale(U: np.ndarray, V: np.ndarray) -> np.ndarray:
    """sum_c |V[pos][bp][c]| |U[pos][c][k]|: the magnitude that bounds the FP32
    rounding of the GEMM's sums in any order."""
    return np.matmul(np.abs(V.astype(np.float64)), np.abs(U.astype(np.float64)))


def input_transform_scale(x: np.ndarray, nh: int, nw: int, pad: int) -> np.ndarray:
    """Sum of the magnitudes of the 16 terms behind each V[pos][bp][c]
    (|B|^T |d| |B|), the scale within_fp32_reordering takes for V."""
    Ba = np.abs(matrices("ref")[1])
    d = np.abs(input_tiles(x, nh, nw, pad)).astype(np.float64)
    v = Ba.T @ d @ Ba
    return v.transpose(4, 5, 0, 2, 3, 1).reshape(64, -1, x.shape[1])


def filter_transform_scale(w: np.ndarray) -> np.ndarray:
    """Sum of the magnitudes of the 9 terms behind each U[pos][c][k]
    (|G| |w| |G|^T), the scale within_fp32_reordering takes for U."""
    Ga = np.abs(matrices("ref")[2])
    u = Ga @ np.abs(w).astype(np.float64) @ Ga.T
    return u.transpose(2, 3, 1, 0).reshape(64, w.shape[1], w.shape[0])


def output_transform_scale(M: np.ndarray, B: int, nh: int, nw: int, Ho: int,
                           Wo: int) -> np.ndarray:
    """Sum of the magnitudes of the terms behind each y[b][k][h][w]
    (|A|^T |M| |A|), the scale within_fp32_reordering takes for y."""
    Aa = np.abs(matrices("ref")[0])
    K = M.shape[2]
    m = np.abs(M.astype(np.float64)).reshape(8, 8, B, nh, nw, K).transpose(2, 5, 3, 4, 0, 1)
    y = (Aa @ m @ Aa.T).transpose(0, 1, 2, 4, 3, 5).reshape(B, K, nh * 6, nw * 6)
    return y[:, :, :Ho, :Wo]


def within_fp32_reordering(a: np.ndarray, b: np.ndarray, scale: np.ndarray,
                           terms: int) -> np.ndarray:
    """True where FP16 results a and b can both come from the same exact value
    by FP32 sums of ``terms`` products taken in different orders and then
    rounded to FP16: |a - b| <= one FP16 ulp at their magnitude plus
    2 * terms * 2^-24 * scale (``scale`` = sum of the terms' magnitudes)."""
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    mag = np.maximum(np.abs(a64), np.abs(b64))
    ulp16 = np.spacing(mag.astype(np.float16)).astype(np.float64)
    return np.abs(a64 - b64) <= ulp16 + 2.0 * terms * 2.0 ** -24 * scale


# ---------------------------------------------------------------------------
# Weight gradient by the same algorithm (checker for nova_weight_grad_v2).
#
# The reference's backward computes grad_weight exactly in FP32 with a
# per-sample unfold loop (nova_winograd/conv2d.py:131-141).  Differentiating
# the forward y = A [(G w G^T) . (B^T d B)] A^T with respect to w gives
# dW = G^T [ sum over tiles (A^T dY A) . (B^T d B) ] G, the exact gradient in
# exact arithmetic; "ref" stores both transforms in FP16 as the kernels do.
# ---------------------------------------------------------------------------

def weight_grad(x: np.ndarray, dy: np.ndarray, pad: int = 1, mode: str = "ref") -> np.ndarray:
    """dW [K][C][3][3] (float32) from x [B][C][H][W] and dy [B][K][H_out][W_out]."""
    A, _, G = matrices(mode)
    Bn, C, H, W = x.shape
    K = dy.shape[1]
    nh, nw = live_tiling(H, W, pad)
    H_out, W_out = H + 2 * pad - 2, W + 2 * pad - 2
    V = input_transform(x, nh, nw, pad, mode)                  # [64][BP][C]
    t = np.zeros((Bn, K, nh * 6, nw * 6), dtype=np.float32)
    t[:, :, :H_out, :W_out] = dy.astype(np.float32)
    t = t.reshape(Bn, K, nh, 6, nw, 6).transpose(0, 1, 2, 4, 3, 5)
    g = A.T @ t @ A                                            # [B, K, nh, nw, 8, 8]
    g = _round(g.transpose(4, 5, 0, 2, 3, 1).reshape(64, Bn * nh * nw, K), mode)
    ug = np.einsum("pbk,pbc->pkc", g.astype(np.float64), V.astype(np.float64))
    dw = np.einsum("nr,nmkc,ms->kcrs", G.astype(np.float64), ug.reshape(8, 8, K, C),
                   G.astype(np.float64))
    return dw.astype(np.float32)


def direct_weight_grad_fp64(x: np.ndarray, dy: np.ndarray, pad: int = 1) -> np.ndarray:
    """The exact weight gradient of the 3x3 stride-1 convolution, in FP64."""
    Bn, C, H, W = x.shape
    H_out, W_out = dy.shape[2], dy.shape[3]
    xp = np.zeros((Bn, C, H + 2 * pad, W + 2 * pad), dtype=np.float64)
    xp[:, :, pad:pad + H, pad:pad + W] = x.astype(np.float64)
    win = np.lib.stride_tricks.sliding_window_view(xp, (3, 3), axis=(2, 3))[:, :, :H_out, :W_out]
    return np.einsum("bkhw,bchwij->kcij", dy.astype(np.float64), win, optimize=True)


# ---------------------------------------------------------------------------
# FP64 direct convolution (the accuracy yardstick) and the error metric.
# ---------------------------------------------------------------------------

def direct_conv_fp64(x: np.ndarray, w: np.ndarray, pad: int = 1) -> np.ndarray:
    Bn, C, H, W = x.shape
    K = w.shape[0]
    xp = np.zeros((Bn, C, H + 2 * pad, W + 2 * pad), dtype=np.float64)
    xp[:, :, pad:pad + H, pad:pad + W] = x.astype(np.float64)
    H_out, W_out = H + 2 * pad - 2, W + 2 * pad - 2
    win = np.lib.stride_tricks.sliding_window_view(xp, (3, 3), axis=(2, 3))[:, :, :H_out, :W_out]
    return np.einsum("bchwij,kcij->bkhw", win, w.astype(np.float64), optimize=True)


def rel_l2(a: np.ndarray, ref: np.ndarray) -> float:
    a = a.astype(np.float64)
    ref = ref.astype(np.float64)
    return float(np.linalg.norm((a - ref).ravel()) / np.linalg.norm(ref.ravel()))


def synthetic_case(B: int, C: int, K: int, H: int, W: int, seed: int):
    """Seeded inputs of the benchmark distributions: x ~ N(0,1) -> FP16,
    w ~ Kaiming-normal (std sqrt(2/(9C))) FP32."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((B, C, H, W), dtype=np.float32).astype(np.float16)
    w = (rng.standard_normal((K, C, 3, 3), dtype=np.float32) * np.float32(np.sqrt(2.0 / (9 * C))))
    return x, w.astype(np.float32)
