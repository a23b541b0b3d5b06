// Shared definitions for the NOVA F(6,3) Winograd library (sm_100a).
//
// NOVA interpolation points {0, +-3/5, +-1, +-7/6, inf}; m = 6 outputs, r = 3 taps,
// tile n = 8.  The transform constants are the reference tables
// (Jayluci4/nova-wino-amd csrc/nova_winograd.hip:68-97).  A and B are used at the
// precision the reference computes with: the reference uploads them as __half
// (csrc/nova_winograd.hip:103-131), so every A/B constant below is the FP16
// rounding of the table entry written as an exact hex-float.  G stays FP32, as in
// the reference.  The symmetric point pairs (+-p) make each 1-D transform an
// even/odd butterfly, which is how the helpers below evaluate it.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace nova {

// ---- B (input transform V = B^T d B), FP16-rounded table entries ----------
constexpr float kB049  = 0x1.f5cp-2f;   // 0.49
constexpr float kB2211 = 0x1.1b0p+1f;   // 2.2111111111
constexpr float kB2721 = 0x1.5c4p+1f;   // 2.7211111111
constexpr float kB1361 = 0x1.5c8p+0f;   // 1.3611111111
constexpr float kB2361 = 0x1.2e4p+1f;   // 2.3611111111
constexpr float kB0817 = 0x1.a24p-1f;   // 0.8166666667
constexpr float kB1417 = 0x1.6acp+0f;   // 1.4166666667
constexpr float kB06   = 0x1.334p-1f;   // 0.6
constexpr float kB1721 = 0x1.b88p+0f;   // 1.7211111111
constexpr float kB036  = 0x1.70cp-2f;   // 0.36
constexpr float kB1360 = 0x1.5c4p+0f;   // 1.36
constexpr float kB042  = 0x1.ae0p-2f;   // 0.42
constexpr float kB1587 = 0x1.964p+0f;   // 1.5866666667
constexpr float kB1167 = 0x1.2acp+0f;   // 1.1666666667

// ---- A (output transform Y = A M A^T), FP16-rounded table entries ---------
constexpr float kA06    = 0x1.334p-1f;  // 0.6
constexpr float kA1167  = 0x1.2acp+0f;  // 1.1666666667
constexpr float kA036   = 0x1.70cp-2f;  // 0.36
constexpr float kA1361  = 0x1.5c8p+0f;  // 1.3611111111
constexpr float kA0216  = 0x1.ba4p-3f;  // 0.216
constexpr float kA1588  = 0x1.968p+0f;  // 1.5879629630
constexpr float kA01296 = 0x1.098p-3f;  // 0.1296
constexpr float kA1853  = 0x1.da4p+0f;  // 1.8526234568
constexpr float kA00778 = 0x1.3e8p-4f;  // 0.07776
constexpr float kA2161  = 0x1.14cp+1f;  // 2.1613940329

// ---- G (filter transform U = G w G^T), FP32 as in the reference -----------
__host__ __device__ constexpr float kG(int i, int j) {
  constexpr float g[8][3] = {
      {-2.0408163265f, 0.0000000000f, 0.0000000000f},
      {2.1677302997f, 1.3006381798f, 0.7803829079f},
      {2.1677302997f, -1.3006381798f, 0.7803829079f},
      {-2.1634615385f, -2.1634615385f, -2.1634615385f},
      {-2.1634615385f, 2.1634615385f, -2.1634615385f},
      {1.0161394021f, 1.1854959691f, 1.3830786306f},
      {1.0161394021f, -1.1854959691f, 1.3830786306f},
      {0.0000000000f, 0.0000000000f, 1.0000000000f}};
  return g[i][j];
}

// f[r] = sum_i B[i][r] v[i]  (one 8-point input-transform pass).
// Column r of B: r=0 (-.49,0,2.21,0,-2.72,0,1,0); r=1/2 = E1 +- O1; r=3/4 =
// E2 +- O2; r=5/6 = E3 +- O3; r=7 (0,-.49,0,2.21,0,-2.72,0,1).
__device__ __forceinline__ void bt_1d(const float v[8], float f[8]) {
  const float e1 = fmaf(kB1361, v[2], fmaf(-kB2361, v[4], v[6]));
  const float o1 = fmaf(kB0817, v[1], fmaf(-kB1417, v[3], kB06 * v[5]));
  const float e2 = fmaf(kB049, v[2], fmaf(-kB1721, v[4], v[6]));
  const float o2 = fmaf(kB049, v[1], fmaf(-kB1721, v[3], v[5]));
  const float e3 = fmaf(kB036, v[2], fmaf(-kB1360, v[4], v[6]));
  const float o3 = fmaf(kB042, v[1], fmaf(-kB1587, v[3], kB1167 * v[5]));
  f[0] = fmaf(-kB049, v[0], fmaf(kB2211, v[2], fmaf(-kB2721, v[4], v[6])));
  f[1] = e1 + o1;
  f[2] = e1 - o1;
  f[3] = e2 + o2;
  f[4] = e2 - o2;
  f[5] = e3 + o3;
  f[6] = e3 - o3;
  f[7] = fmaf(-kB049, v[1], fmaf(kB2211, v[3], fmaf(-kB2721, v[5], v[7])));
}

// bt_1d split in two halves of its outputs with exactly its operations: rows
// {0, 1, 2, 7} and rows {3, 4, 5, 6}.
__device__ __forceinline__ void bt_1d_a(const float v[8], float f[4]) {
  const float e1 = fmaf(kB1361, v[2], fmaf(-kB2361, v[4], v[6]));
  const float o1 = fmaf(kB0817, v[1], fmaf(-kB1417, v[3], kB06 * v[5]));
  f[0] = fmaf(-kB049, v[0], fmaf(kB2211, v[2], fmaf(-kB2721, v[4], v[6])));
  f[1] = e1 + o1;
  f[2] = e1 - o1;
  f[3] = fmaf(-kB049, v[1], fmaf(kB2211, v[3], fmaf(-kB2721, v[5], v[7])));
}
__device__ __forceinline__ void bt_1d_b(const float v[8], float f[4]) {
  const float e2 = fmaf(kB049, v[2], fmaf(-kB1721, v[4], v[6]));
  const float o2 = fmaf(kB049, v[1], fmaf(-kB1721, v[3], v[5]));
  const float e3 = fmaf(kB036, v[2], fmaf(-kB1360, v[4], v[6]));
  const float o3 = fmaf(kB042, v[1], fmaf(-kB1587, v[3], kB1167 * v[5]));
  f[0] = e2 + o2;
  f[1] = e2 - o2;
  f[2] = e3 + o3;
  f[3] = e3 - o3;
}

// A[i][p] (6 x 8, FP16-rounded entries) as a table, for code that indexes A
// rather than running the butterfly.
__host__ __device__ constexpr float kA(int i, int p) {
  constexpr float a[6][8] = {
      {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 0.f},
      {0.f, kA06, -kA06, 1.f, -1.f, kA1167, -kA1167, 0.f},
      {0.f, kA036, kA036, 1.f, 1.f, kA1361, kA1361, 0.f},
      {0.f, kA0216, -kA0216, 1.f, -1.f, kA1588, -kA1588, 0.f},
      {0.f, kA01296, kA01296, 1.f, 1.f, kA1853, kA1853, 0.f},
      {0.f, kA00778, -kA00778, 1.f, -1.f, kA2161, -kA2161, 1.f}};
  return a[i][p];
}

// g[i] = sum_p A[i][p] m[p]  (one 8 -> 6 output-transform pass).
__device__ __forceinline__ void a_1d(const float m[8], float g[6]) {
  const float sa = m[1] + m[2], da = m[1] - m[2];
  const float sb = m[3] + m[4], db = m[3] - m[4];
  const float sc = m[5] + m[6], dc = m[5] - m[6];
  g[0] = m[0] + sa + sb + sc;
  g[1] = fmaf(kA06, da, fmaf(kA1167, dc, db));
  g[2] = fmaf(kA036, sa, fmaf(kA1361, sc, sb));
  g[3] = fmaf(kA0216, da, fmaf(kA1588, dc, db));
  g[4] = fmaf(kA01296, sa, fmaf(kA1853, sc, sb));
  g[5] = fmaf(kA00778, da, fmaf(kA2161, dc, db)) + m[7];
}

// ---- Programmatic dependent launch ---------------------------------------
// Hot-path kernels are launched with programmatic stream serialization, so a
// kernel may start while its predecessor in the stream is still finishing.
// pdl_wait() blocks until the predecessor grid has completed and its memory
// is visible; every such kernel calls it before its first global-memory
// access (read or write).  pdl_trigger() lets the successor start launching
// once every CTA of this grid has called it (or exited).  Both are no-ops for
// a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- Paired-lane forms (sm_100 FFMA2 / FADD2 / FMUL2) ----------------------
// The same butterflies on two independent values at once (two channels).  Each
// component goes through exactly the operations of bt_1d / a_1d in the same
// order with the same rounding, so results are bit-identical to the scalar
// forms; the paired instructions halve the FP32 instruction count.
__device__ __forceinline__ float2 bc2(float k) { return make_float2(k, k); }
__device__ __forceinline__ float2 fma2(float k, float2 a, float2 b) {
  return __ffma2_rn(bc2(k), a, b);
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  return __fadd2_rn(a, make_float2(-b.x, -b.y));
}
__device__ __forceinline__ float2 mul2(float k, float2 a) { return __fmul2_rn(bc2(k), a); }

__device__ __forceinline__ void bt_1d2(const float2 v[8], float2 f[8]) {
  const float2 e1 = fma2(kB1361, v[2], fma2(-kB2361, v[4], v[6]));
  const float2 o1 = fma2(kB0817, v[1], fma2(-kB1417, v[3], mul2(kB06, v[5])));
  const float2 e2 = fma2(kB049, v[2], fma2(-kB1721, v[4], v[6]));
  const float2 o2 = fma2(kB049, v[1], fma2(-kB1721, v[3], v[5]));
  const float2 e3 = fma2(kB036, v[2], fma2(-kB1360, v[4], v[6]));
  const float2 o3 = fma2(kB042, v[1], fma2(-kB1587, v[3], mul2(kB1167, v[5])));
  f[0] = fma2(-kB049, v[0], fma2(kB2211, v[2], fma2(-kB2721, v[4], v[6])));
  f[1] = add2(e1, o1);
  f[2] = sub2(e1, o1);
  f[3] = add2(e2, o2);
  f[4] = sub2(e2, o2);
  f[5] = add2(e3, o3);
  f[6] = sub2(e3, o3);
  f[7] = fma2(-kB049, v[1], fma2(kB2211, v[3], fma2(-kB2721, v[5], v[7])));
}

// bt_1d2 split in two halves of its outputs, with exactly its operations:
// rows {0, 1, 2, 7} and rows {3, 4, 5, 6}.  A 2-D transform that keeps only one
// half of the column pass live at a time needs 64 registers instead of 128.
__device__ __forceinline__ void bt_1d2_a(const float2 v[8], float2 f[4]) {
  const float2 e1 = fma2(kB1361, v[2], fma2(-kB2361, v[4], v[6]));
  const float2 o1 = fma2(kB0817, v[1], fma2(-kB1417, v[3], mul2(kB06, v[5])));
  f[0] = fma2(-kB049, v[0], fma2(kB2211, v[2], fma2(-kB2721, v[4], v[6])));
  f[1] = add2(e1, o1);
  f[2] = sub2(e1, o1);
  f[3] = fma2(-kB049, v[1], fma2(kB2211, v[3], fma2(-kB2721, v[5], v[7])));
}
__device__ __forceinline__ void bt_1d2_b(const float2 v[8], float2 f[4]) {
  const float2 e2 = fma2(kB049, v[2], fma2(-kB1721, v[4], v[6]));
  const float2 o2 = fma2(kB049, v[1], fma2(-kB1721, v[3], v[5]));
  const float2 e3 = fma2(kB036, v[2], fma2(-kB1360, v[4], v[6]));
  const float2 o3 = fma2(kB042, v[1], fma2(-kB1587, v[3], mul2(kB1167, v[5])));
  f[0] = add2(e2, o2);
  f[1] = sub2(e2, o2);
  f[2] = add2(e3, o3);
  f[3] = sub2(e3, o3);
}

// ---- Butterflies over inputs known to be zero ------------------------------
// A tile whose window reaches past the image's last row (or column) has
// inputs v[i] = 0 for i >= N.  Zv carries a value with a flag that is a
// compile-time constant once the butterfly is unrolled; a term whose input is
// known zero is dropped (fma(k, 0, c) == c), and an FMA onto a known-zero
// accumulator becomes a multiply (fma(k, a, 0) == k * a, one rounding both
// ways).  The remaining operations run in bt_1d2's order, so every output
// equals bt_1d2's except possibly in the sign of an exact zero.
struct Zv {
  float2 v;
  bool on;  // false: the value is known to be zero
};
__device__ __forceinline__ Zv zin(const float2* v, int i, int n) {
  return i < n ? Zv{v[i], true} : Zv{make_float2(0.f, 0.f), false};
}
__device__ __forceinline__ Zv zmul(float k, Zv a) { return a.on ? Zv{mul2(k, a.v), true} : a; }
__device__ __forceinline__ Zv zfma(float k, Zv a, Zv c) {
  if (!a.on) return c;
  if (!c.on) return Zv{mul2(k, a.v), true};
  return Zv{fma2(k, a.v, c.v), true};
}
__device__ __forceinline__ float2 zadd(Zv a, Zv b) {
  if (!a.on) return b.on ? b.v : make_float2(0.f, 0.f);
  if (!b.on) return a.v;
  return add2(a.v, b.v);
}
__device__ __forceinline__ float2 zsub(Zv a, Zv b) {
  if (!b.on) return a.on ? a.v : make_float2(0.f, 0.f);
  if (!a.on) return make_float2(-b.v.x, -b.v.y);
  return sub2(a.v, b.v);
}
__device__ __forceinline__ float2 zval(Zv a) { return a.on ? a.v : make_float2(0.f, 0.f); }

// bt_1d2 / bt_1d2_a / bt_1d2_b with v[i] = 0 for i >= N (N = 8: the same
// operations as the dense forms).
template <int N>
__device__ __forceinline__ void bt_1d2_za(const float2 v[8], float2 f[4]) {
  const Zv v0 = zin(v, 0, N), v1 = zin(v, 1, N), v2 = zin(v, 2, N), v3 = zin(v, 3, N);
  const Zv v4 = zin(v, 4, N), v5 = zin(v, 5, N), v6 = zin(v, 6, N), v7 = zin(v, 7, N);
  const Zv e1 = zfma(kB1361, v2, zfma(-kB2361, v4, v6));
  const Zv o1 = zfma(kB0817, v1, zfma(-kB1417, v3, zmul(kB06, v5)));
  f[0] = zval(zfma(-kB049, v0, zfma(kB2211, v2, zfma(-kB2721, v4, v6))));
  f[1] = zadd(e1, o1);
  f[2] = zsub(e1, o1);
  f[3] = zval(zfma(-kB049, v1, zfma(kB2211, v3, zfma(-kB2721, v5, v7))));
}
template <int N>
__device__ __forceinline__ void bt_1d2_zb(const float2 v[8], float2 f[4]) {
  const Zv v1 = zin(v, 1, N), v2 = zin(v, 2, N), v3 = zin(v, 3, N);
  const Zv v4 = zin(v, 4, N), v5 = zin(v, 5, N), v6 = zin(v, 6, N);
  const Zv e2 = zfma(kB049, v2, zfma(-kB1721, v4, v6));
  const Zv o2 = zfma(kB049, v1, zfma(-kB1721, v3, v5));
  const Zv e3 = zfma(kB036, v2, zfma(-kB1360, v4, v6));
  const Zv o3 = zfma(kB042, v1, zfma(-kB1587, v3, zmul(kB1167, v5)));
  f[0] = zadd(e2, o2);
  f[1] = zsub(e2, o2);
  f[2] = zadd(e3, o3);
  f[3] = zsub(e3, o3);
}
template <int N>
__device__ __forceinline__ void bt_1d2_z(const float2 v[8], float2 f[8]) {
  float2 a[4], b[4];
  bt_1d2_za<N>(v, a);
  bt_1d2_zb<N>(v, b);
  f[0] = a[0];
  f[1] = a[1];
  f[2] = a[2];
  f[3] = b[0];
  f[4] = b[1];
  f[5] = b[2];
  f[6] = b[3];
  f[7] = a[3];
}

__device__ __forceinline__ void a_1d2(const float2 m[8], float2 g[6]) {
  const float2 sa = add2(m[1], m[2]), da = sub2(m[1], m[2]);
  const float2 sb = add2(m[3], m[4]), db = sub2(m[3], m[4]);
  const float2 sc = add2(m[5], m[6]), dc = sub2(m[5], m[6]);
  g[0] = add2(add2(add2(m[0], sa), sb), sc);
  g[1] = fma2(kA06, da, fma2(kA1167, dc, db));
  g[2] = fma2(kA036, sa, fma2(kA1361, sc, sb));
  g[3] = fma2(kA0216, da, fma2(kA1588, dc, db));
  g[4] = fma2(kA01296, sa, fma2(kA1853, sc, sb));
  g[5] = add2(fma2(kA00778, da, fma2(kA2161, dc, db)), m[7]);
}

}  // namespace nova
