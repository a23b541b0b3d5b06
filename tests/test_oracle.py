"""CPU tests of the oracle: pinned against the reference's own tables, its
compiled compute_tiling, its published error figure, and a per-thread
pure-Python restatement of its kernels (small sizes)."""

import json
import os

import numpy as np
import pytest

import nova_oracle as o

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    with open(os.path.join(GOLDEN, name)) as f:
        return json.load(f)


def test_matrices_match_reference_tables():
    g = _load("nova_matrices.json")
    np.testing.assert_array_equal(np.array(g["A"]), o.A_TABLE)
    np.testing.assert_array_equal(np.array(g["B"]), o.B_TABLE)
    np.testing.assert_array_equal(np.array(g["G"]), o.G_TABLE)


def test_cook_toom_identity():
    # The tables realise the F(6,3) minimal filtering identity (to the 1e-10
    # precision they are printed with).
    assert o.cook_toom_residual() < 1e-8


def test_tiling_matches_compiled_reference():
    rows = _load("tiling.json")["rows"]
    assert len(rows) > 700
    for H, W, pad, nh, nw, Ho, Wo in rows:
        assert o.compute_tiling(H, W, pad) == (nh, nw, Ho, Wo), (H, W, pad)


def test_tiling_known_stage_values():
    # H -> nh for the ResNet stage sizes (reference over-tiles by one or two).
    for H, nh in [(56, 11), (28, 6), (14, 4), (7, 2), (64, 12), (32, 7), (128, 23), (16, 4), (224, 39)]:
        assert o.compute_tiling(H, H, 1)[0] == nh
    for H in range(1, 300):
        live = o.live_tiling(H, H, 1)[0]
        assert live == -(-H // 6)
        assert live <= o.compute_tiling(H, H, 1)[0]


def test_published_fp16_error_reproduced():
    # docs/report/main.tex:217: NOVA F(6,3) FP16 relative error vs FP32 direct = 5.2 %.
    known = _load("known_answers.json")["fp16_rel_error_vs_fp32_direct"]["value"]
    x, w = o.synthetic_case(1, 64, 64, 56, 56, seed=1234)
    err = o.rel_l2(o.nova_forward(x, w, 1, "ref"), o.direct_conv_fp64(x, w, 1))
    assert abs(err - known) < 0.004, err


def test_exact_mode_is_fp32_accurate():
    x, w = o.synthetic_case(1, 64, 64, 28, 28, seed=7)
    err = o.rel_l2(o.nova_forward(x, w, 1, "exact"), o.direct_conv_fp64(x, w, 1))
    assert err < 1e-4


@pytest.mark.parametrize("B,C,K,H", [(1, 64, 64, 56), (1, 128, 128, 28), (1, 256, 256, 14), (2, 16, 24, 20)])
def test_ref_mode_within_reference_tolerance(B, C, K, H):
    tol = _load("known_answers.json")["test_rel_l2_tolerance"]["value"]
    x, w = o.synthetic_case(B, C, K, H, H, seed=B * 1000 + C)
    y = o.nova_forward(x, w, 1, "ref")
    assert np.isfinite(y.astype(np.float32)).all()
    assert o.rel_l2(y, o.direct_conv_fp64(x, w, 1)) < tol


def test_dead_tiles_change_nothing():
    x, w = o.synthetic_case(2, 8, 8, 56, 44, seed=3)
    a = o.nova_forward(x, w, 1, "ref", live_tiles_only=True)
    b = o.nova_forward(x, w, 1, "ref", live_tiles_only=False)
    np.testing.assert_array_equal(a, b)


# ---------------------------------------------------------------------------
# Per-thread restatement of the reference kernels (pure Python, tiny sizes),
# following their index arithmetic literally, to pin the oracle's layouts.
# ---------------------------------------------------------------------------

def _ref_input_transform_loops(x, nh, nw, pad, BP):
    """input_transform_kernel, csrc/nova_winograd.hip:141-205 (one block per tile)."""
    A, Bm, _ = o.matrices("ref")
    Bn, C, H, W = x.shape
    P = nh * nw
    V = np.zeros(64 * C * BP, dtype=np.float16)
    for gi in range(Bn * C * P):
        b, rem = divmod(gi, C * P)
        c, tile = divmod(rem, P)
        th, tw = divmod(tile, nw)
        hs, ws = th * 6 - pad, tw * 6 - pad
        t = np.zeros((8, 8), np.float32)
        for r in range(8):
            for cc in range(8):
                hi, wi = hs + r, ws + cc
                if 0 <= hi < H and 0 <= wi < W:
                    t[r, cc] = np.float32(x[b, c, hi, wi])
        temp = np.zeros((8, 8), np.float32)
        for r in range(8):
            for cc in range(8):
                s = np.float32(0)
                for k in range(8):
                    s = np.float32(s + Bm[k, r] * t[k, cc])      # c_BT[row][k] = B[k][row]
                temp[r, cc] = s
        for r in range(8):
            for cc in range(8):
                s = np.float32(0)
                for k in range(8):
                    s = np.float32(s + temp[r, k] * Bm[k, cc])
                bp = b * P + tile
                V[(r * 8 + cc) * C * BP + c + bp * C] = np.float16(s)
    return V.reshape(64, BP, C)


def _ref_output_transform_loops(M, Bn, K, H_out, W_out, nh, nw, BP):
    """output_transform_kernel, csrc/nova_winograd.hip:264-328."""
    A, _, _ = o.matrices("ref")
    P = nh * nw
    Mf = M.reshape(-1)
    y = np.zeros((Bn, K, H_out, W_out), np.float16)
    for gi in range(Bn * K * P):
        b, rem = divmod(gi, K * P)
        k, tile = divmod(rem, P)
        th, tw = divmod(tile, nw)
        bp = b * P + tile
        m = np.array([[np.float32(Mf[(r * 8 + c) * K * BP + k + bp * K]) for c in range(8)]
                      for r in range(8)], np.float32)
        temp = np.zeros((6, 8), np.float32)
        for r in range(6):
            for c in range(8):
                s = np.float32(0)
                for p in range(8):
                    s = np.float32(s + A[r, p] * m[p, c])
                temp[r, c] = s
        for r in range(6):
            for c in range(6):
                s = np.float32(0)
                for p in range(8):
                    s = np.float32(s + temp[r, p] * A[c, p])
                ho, wo = th * 6 + r, tw * 6 + c
                if ho < H_out and wo < W_out:
                    y[b, k, ho, wo] = np.float16(s)
    return y


def _ref_filter_transform_loops(w):
    """filter_transform_kernel, csrc/nova_winograd.hip:214-255."""
    _, _, G = o.matrices("ref")
    K, C = w.shape[:2]
    U = np.zeros(64 * K * C, np.float16)
    for gi in range(K * C):
        k, c = divmod(gi, C)
        for r in range(8):
            for cc in range(8):
                s = np.float32(0)
                for p in range(3):
                    for q in range(3):
                        s = np.float32(s + G[r, p] * np.float32(w[k, c, p, q]) * G[cc, q])
                U[(r * 8 + cc) * K * C + k + c * K] = np.float16(s)
    return U.reshape(64, C, K)


def _ulp_close(a, b, max_ulp=1):
    ai = a.astype(np.float16).view(np.int16).astype(np.int32)
    bi = b.astype(np.float16).view(np.int16).astype(np.int32)
    return np.abs(ai - bi).max() <= max_ulp


def test_oracle_layouts_match_reference_kernel_loops():
    x, w = o.synthetic_case(2, 3, 2, 9, 7, seed=11)
    pad = 1
    nh, nw, Ho, Wo = o.compute_tiling(9, 7, pad)
    BP = 2 * nh * nw
    V_loop = _ref_input_transform_loops(x, nh, nw, pad, BP)
    V_vec = o.input_transform(x, nh, nw, pad, "ref")
    assert V_vec.shape == V_loop.shape
    assert _ulp_close(V_vec, V_loop)
    U_loop = _ref_filter_transform_loops(w)
    U_vec = o.filter_transform(w, "ref")
    assert _ulp_close(U_vec, U_loop)
    M = o.gemm(U_vec, V_vec, "ref")
    y_loop = _ref_output_transform_loops(M, 2, 2, Ho, Wo, nh, nw, BP)
    y_vec = o.output_transform(M, 2, nh, nw, Ho, Wo, "ref")
    assert _ulp_close(y_vec, y_loop)


def test_exact_order_restatement_agrees_with_fast_oracle():
    """The *_seq functions (the reference kernels' FMA chains in order) and the
    vectorised "ref" functions differ only by FP32 summation order."""
    x, w = o.synthetic_case(2, 8, 12, 11, 13, seed=9)
    nh, nw, Ho, Wo = o.compute_tiling(11, 13, 1)
    U, Us = o.filter_transform(w, "ref"), o.filter_transform_seq(w)
    assert U.shape == Us.shape
    _, _, G = o.matrices("ref")
    sc = np.abs(G) @ np.abs(w).astype(np.float64) @ np.abs(G).T
    sc = sc.transpose(2, 3, 1, 0).reshape(64, 8, 12)
    assert o.within_fp32_reordering(Us, U, sc, 9).all()
    V, Vs = o.input_transform(x, nh, nw, 1, "ref"), o.input_transform_seq(x, nh, nw, 1)
    assert V.shape == Vs.shape and o.rel_l2(Vs, V) < 1e-3
    M = o.gemm(U, V, "ref")
    y, ys = o.output_transform(M, 2, nh, nw, Ho, Wo, "ref"), o.output_transform_seq(M, 2, nh, nw, Ho, Wo)
    assert y.shape == ys.shape and o.rel_l2(ys, y) < 1e-3
    # The reordering predicate rejects a real difference.
    bad = ys.copy()
    bad[0, 0, 0, 0] = np.float16(float(bad[0, 0, 0, 0]) + 0.5)
    assert not o.within_fp32_reordering(bad, ys, np.zeros(ys.shape), 16).all()


def test_weight_grad_identity():
    """dW = G^T [sum over tiles (A^T dY A) . (B^T d B)] G is the exact weight
    gradient: in the "exact" mode it matches the FP64 direct gradient (ragged
    tiles and pad 0 included); with the FP16 storage of the transforms its error
    is of the order of the forward's."""
    rng = np.random.default_rng(1)
    for (B, C, K, H, W, pad) in [(2, 16, 24, 13, 17, 1), (1, 8, 8, 10, 9, 0)]:
        x = rng.standard_normal((B, C, H, W)).astype(np.float16)
        dy = rng.standard_normal((B, K, H + 2 * pad - 2, W + 2 * pad - 2)).astype(np.float16)
        d = o.direct_weight_grad_fp64(x, dy, pad)
        assert o.rel_l2(o.weight_grad(x, dy, pad, "exact"), d) < 1e-4
        assert o.rel_l2(o.weight_grad(x, dy, pad, "ref"), d) < 0.08
