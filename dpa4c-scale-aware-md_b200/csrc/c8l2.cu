// C8L2 profile kernels (see c8l2.cuh).
//
// Layout of the 40 moments of a node (Profile<8, 2, false> of the reference,
// include/dpa_chain/graph_compress_launch.h:318-334): scalars [0, 8), degree
// one [8, 20) as [component 3][channel 4], degree two [20, 40) as
// [component 5][channel 4].  The 70 descriptor entries
// (graph_compress_launch.h:346-381): scalars [0, 8), Gram of the aligned
// degree-one block [8, 18), Gram of the aligned degree-two block [18, 28),
// bispectrum 112 [28, 48), bispectrum 222 [48, 52), quartic [52, 60), the two
// moment divisors [60, 62), the centre's type embedding [62, 70); each stored
// as (value - mean) * inv_std.
#include <algorithm>
#include <cmath>
#include <type_traits>

#include "c8l2.cuh"
#include "common.cuh"
#include "simt_gemm.cuh"

namespace b200dp {

namespace {

constexpr int kC8Warps = 8;
constexpr int kMom = 40;
constexpr int kVec = 8, kTen = 20;  // moment offsets of degree one and two

template <typename P>
struct C8V {
  int T, nint, act;
  P stride, rcut, eps2, floor_;
  const P* table;
  const P* film;
  const P* temb;
  const P* ro;
  const P* mean;
  const P* istd;
  __host__ __device__ explicit C8V(const C8Dev& d)
      : T(d.ntypes), nint(d.nint), act(d.act), stride((P)d.stride), rcut((P)d.rcut), eps2((P)(d.eps * d.eps)),
        floor_((P)d.floor_), table(static_cast<const P*>(d.table)), film(static_cast<const P*>(d.film)),
        temb(static_cast<const P*>(d.temb)), ro(static_cast<const P*>(d.readout)),
        mean(static_cast<const P*>(d.mean)), istd(static_cast<const P*>(d.istd)) {}
  // readout matrix k, entry [row][column]
  __device__ __forceinline__ P R(int k, int r, int c) const { return __ldg(ro + k * 16 + r * 4 + c); }
};

template <typename P>
struct Geo {
  P u[3], iR, R, env, denv, b[9], x;
  int idx;
};

// Regularized distance and direction, C3 envelope and its derivative, l <= 2
// harmonics on the unit direction and the canonical table location
// (include/dpa_chain/graph_compress.cuh:97-106, 218-266, 292-304).
template <typename P>
__device__ __forceinline__ Geo<P> c8_geometry(const C8V<P>& m, const double* __restrict__ r) {
  Geo<P> g;
  const P rx = (P)r[0], ry = (P)r[1], rz = (P)r[2];
  const P sq = rx * rx + ry * ry + rz * rz + m.eps2;
  g.R = sqrt(sq);
  g.iR = (P)1 / g.R;
  g.u[0] = rx * g.iR;
  g.u[1] = ry * g.iR;
  g.u[2] = rz * g.iR;
  const P uu = fmin(fmax((m.rcut - g.R) / m.rcut, (P)0), (P)1), xx = (P)1 - uu;
  const P s = (P)1 + xx * ((P)4 + xx * ((P)10 + xx * ((P)20 + (P)35 * xx)));
  const P u2 = uu * uu;
  g.env = u2 * u2 * s;
  if (g.R <= (P)0 || g.R >= m.rcut) {
    g.denv = 0;
  } else {
    const P ds = (P)4 + xx * ((P)20 + xx * ((P)60 + (P)140 * xx));
    g.denv = (-(P)4 * u2 * uu * s + u2 * u2 * ds) / m.rcut;
  }
  const P x = g.u[0], y = g.u[1], z = g.u[2];
  const P s3 = (P)1.7320508075688772935;
  g.b[0] = 1;
  g.b[1] = x;
  g.b[2] = y;
  g.b[3] = z;
  g.b[4] = s3 * x * y;
  g.b[5] = s3 * y * z;
  g.b[6] = (P)0.5 * ((P)3 * z * z - (P)1);
  g.b[7] = s3 * x * z;
  g.b[8] = (P)0.5 * s3 * (x * x - y * y);
  int idx = (int)(g.R / m.stride);
  g.idx = idx < m.nint - 1 ? idx : m.nint - 1;
  g.x = g.R - (P)g.idx * m.stride;
  return g;
}

// Six quintic coefficients of channel c from an interval row.
__device__ __forceinline__ void table_coeffs(const float* row, int c, float (&k)[6]) {
  const float4 q = __ldg(reinterpret_cast<const float4*>(row) + c);
  const float2 p = __ldg(reinterpret_cast<const float2*>(row + 32) + c);
  k[0] = q.x, k[1] = q.y, k[2] = q.z, k[3] = q.w, k[4] = p.x, k[5] = p.y;
}
__device__ __forceinline__ void table_coeffs(const double* row, int c, double (&k)[6]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) k[j] = __ldg(row + 4 * c + j);
  k[4] = __ldg(row + 32 + 2 * c);
  k[5] = __ldg(row + 33 + 2 * c);
}

template <typename P>
__device__ __forceinline__ P poly(const P (&k)[6], P x) {
  return k[0] + (k[1] + (k[2] + (k[3] + (k[4] + k[5] * x) * x) * x) * x) * x;
}
template <typename P>
__device__ __forceinline__ P dpoly(const P (&k)[6], P x) {
  return k[1] + ((P)2 * k[2] + ((P)3 * k[3] + ((P)4 * k[4] + (P)5 * k[5] * x) * x) * x) * x;
}

template <typename P>
__device__ __forceinline__ P wsum(P v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// decode_upper_pair of the reference (graph_compress.cuh:638-647)
__device__ __forceinline__ void upper_pair(int pair, int width, int& r, int& c) {
  r = 0;
  while (pair >= width - r) {
    pair -= width - r;
    ++r;
  }
  c = r + pair;
}
__device__ __forceinline__ int pair_pos(int a, int b, int width) {
  const int r = a < b ? a : b, c = a < b ? b : a;
  return r * width - r * (r - 1) / 2 + c - r;
}

// Symmetric traceless matrix of five packed components and the inverse map
// of a matrix gradient (graph_compress.cuh:565-626).
template <typename P>
__device__ __forceinline__ void stf(const P* p, P (&M)[3][3]) {
  const P is2 = (P)0.7071067811865475244, is6 = (P)0.4082482904638630164;
  M[0][0] = -p[2] * is6 + p[4] * is2;
  M[1][1] = -p[2] * is6 - p[4] * is2;
  M[2][2] = (P)2 * p[2] * is6;
  M[0][1] = M[1][0] = p[0] * is2;
  M[1][2] = M[2][1] = p[1] * is2;
  M[0][2] = M[2][0] = p[3] * is2;
}
template <typename P>
__device__ __forceinline__ void stf_grad(const P (&M)[3][3], P (&g)[5]) {
  const P is2 = (P)0.7071067811865475244, is6 = (P)0.4082482904638630164;
  g[0] = (M[0][1] + M[1][0]) * is2;
  g[1] = (M[1][2] + M[2][1]) * is2;
  g[2] = (-M[0][0] - M[1][1] + (P)2 * M[2][2]) * is6;
  g[3] = (M[0][2] + M[2][0]) * is2;
  g[4] = (M[0][0] - M[1][1]) * is2;
}
template <typename P>
__device__ __forceinline__ void mat_mul(const P (&A)[3][3], const P (&B)[3][3], P (&C)[3][3]) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) C[i][j] = A[i][0] * B[0][j] + A[i][1] * B[1][j] + A[i][2] * B[2][j];
}
template <typename P>
__device__ __forceinline__ void mat_vec(const P (&A)[3][3], const P (&v)[3], P (&o)[3]) {
#pragma unroll
  for (int i = 0; i < 3; ++i) o[i] = A[i][0] * v[0] + A[i][1] * v[1] + A[i][2] * v[2];
}

// Per-warp node workspace (shared memory), indices:
// w[0, 40): the 40 normalized moments
constexpr int kW_AV = 40;  // aligned degree one [3][4]
constexpr int kW_AT = 52;  // aligned degree two [5][4]
constexpr int kW_PV = 72;  // degree-one probes [3][4]
constexpr int kW_PT = 84;  // degree-two probes [5][2]
constexpr int kW_MS = 94;  // scalar and angular envelope masses
constexpr int kW_FWD = 96;

// Alignment and probe projections of the normalized moments in w[0, 40)
// (forward step 4, graph_compress_kernel.cuh:482-535): aligned value per lane
// < 32, then probe per lane < 22.
template <typename P>
__device__ __forceinline__ void align_and_probe(const C8V<P>& m, P* w, int lane) {
  P v = 0;
  if (lane < 12) {
    const int comp = lane >> 2, ch = lane & 3;
#pragma unroll
    for (int in = 0; in < 4; ++in) v += w[kVec + comp * 4 + in] * m.R(0, in, ch);
  } else {
    const int l2 = lane - 12, comp = l2 >> 2, ch = l2 & 3;
#pragma unroll
    for (int in = 0; in < 4; ++in) v += w[kTen + comp * 4 + in] * m.R(2, in, ch);
  }
  w[kW_AV + lane] = v;
  __syncwarp();
  if (lane < 22) {
    v = 0;
    if (lane < 12) {
      const int comp = lane >> 2, k = lane & 3;
#pragma unroll
      for (int in = 0; in < 4; ++in) v += w[kW_AV + comp * 4 + in] * m.R(4, in, k);
    } else {
      const int l2 = lane - 12, comp = l2 >> 1, k = l2 & 1;
#pragma unroll
      for (int in = 0; in < 4; ++in) v += w[kW_AT + comp * 4 + in] * m.R(6, in, k);
    }
    w[kW_PV + lane] = v;
  }
  __syncwarp();
}

template <typename P>
__device__ __forceinline__ void probe_vec(const P* w, int k, P (&v)[3]) {
#pragma unroll
  for (int c = 0; c < 3; ++c) v[c] = w[kW_PV + c * 4 + k];
}
template <typename P>
__device__ __forceinline__ void probe_stf(const P* w, int t, P (&Q)[3][3]) {
  P p[5];
#pragma unroll
  for (int c = 0; c < 5; ++c) p[c] = w[kW_PT + c * 2 + t];
  stf(p, Q);
}

// One descriptor entry before the output normalization (forward step 5,
// graph_compress_kernel.cuh:537-700).
template <typename P>
__device__ P c8_output(const C8V<P>& m, const P* w, int o, int ti) {
  const P s2 = (P)1.4142135623730950488, s3 = (P)1.7320508075688772935, is5 = (P)0.44721359549995793928;
  if (o < 8) return w[o];
  if (o < 28) {
    const bool one = o < 18;
    int r, c;
    upper_pair(one ? o - 8 : o - 18, 4, r, c);
    P s = 0;
    if (one) {
#pragma unroll
      for (int k = 0; k < 3; ++k) s += w[kW_AV + k * 4 + r] * w[kW_AV + k * 4 + c];
    } else {
#pragma unroll
      for (int k = 0; k < 5; ++k) s += w[kW_AT + k * 4 + r] * w[kW_AT + k * 4 + c];
    }
    return (r == c ? (P)1 : s2) * s;
  }
  if (o < 48) {
    const int out = o - 28, t = out & 1;
    int a, b;
    upper_pair(out >> 1, 4, a, b);
    P Q[3][3], va[3], vb[3], qb[3];
    probe_stf(w, t, Q);
    probe_vec(w, a, va);
    probe_vec(w, b, vb);
    mat_vec(Q, vb, qb);
    return (a == b ? (P)1 : s2) * (-is5) * (va[0] * qb[0] + va[1] * qb[1] + va[2] * qb[2]);
  }
  if (o < 52) {
    const int k = o - 48;  // entries {000, 001, 011, 111}
    P Q0[3][3], Q1[3][3], AB[3][3], ABC[3][3];
    probe_stf(w, 0, Q0);
    probe_stf(w, 1, Q1);
    mat_mul(k == 3 ? Q1 : Q0, k >= 2 ? Q1 : Q0, AB);
    mat_mul(AB, k >= 1 ? Q1 : Q0, ABC);
    const P sc = (k == 1 || k == 2) ? s3 : (P)1;
    return (P)-0.58554004376911988 * sc * (ABC[0][0] + ABC[1][1] + ABC[2][2]);
  }
  if (o < 60) {
    const int out = o - 52, vi = out & 3, t = out >> 2;
    P Q[3][3], v[3], qv[3];
    probe_stf(w, t, Q);
    probe_vec(w, vi, v);
    mat_vec(Q, v, qv);
    return qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2];
  }
  if (o < 62) return sqrt(w[kW_MS + (o - 60)] + m.floor_);
  return __ldg(m.temb + ti * 8 + (o - 62));
}

// One warp per centre: lanes stride over the centre's slots, each lane
// accumulating all 40 moments and both envelope masses of its edges in
// registers; an xor-tree warp sum (fixed order) merges them, then the node
// readout runs across the lanes on a per-warp shared-memory workspace.
template <typename P>
__global__ void __launch_bounds__(kC8Warps * 32)
    k_c8_forward(C8Dev d, int nloc, int selt, const int* __restrict__ nl_j, const double* __restrict__ rij,
                 const int* __restrict__ atype, P* __restrict__ desc, P* __restrict__ state) {
  __shared__ P ws[kC8Warps][kW_FWD];
  const C8V<P> m(d);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kC8Warps + warp;
  if (i >= nloc) return;  // warp-uniform; only warp-level barriers follow
  const int ti = atype[i];
  P* w = ws[warp];
  P acc[kMom + 2];
#pragma unroll
  for (int k = 0; k < kMom + 2; ++k) acc[k] = 0;
  if (ti >= 0 && ti < m.T) {
    const size_t row = (size_t)i * selt;
    for (int s = lane; s < selt; s += 32) {
      const int j = nl_j[row + s];
      if (j < 0) continue;
      const Geo<P> g = c8_geometry(m, rij + 3 * (row + s));
      const P* film = m.film + ((size_t)ti * m.T + atype[j]) * 16;
      const P* trow = m.table + (size_t)g.idx * 48;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        P k[6];
        table_coeffs(trow, c, k);
        const P f = __ldg(film + 2 * c) * poly(k, g.x) + __ldg(film + 2 * c + 1);
        const P amp = f * g.env, ang = amp * g.env;
        acc[c] += amp;
        if (c < 4) {
#pragma unroll
          for (int q = 0; q < 3; ++q) acc[kVec + q * 4 + c] += ang * g.b[1 + q];
#pragma unroll
          for (int q = 0; q < 5; ++q) acc[kTen + q * 4 + c] += ang * g.b[4 + q];
        }
      }
      const P e2 = g.env * g.env;
      acc[kMom] += e2;
      acc[kMom + 1] += e2 * e2;
    }
  }
#pragma unroll
  for (int k = 0; k < kMom + 2; ++k) acc[k] = wsum(acc[k]);
  const P ns = (P)1 / sqrt(acc[kMom] + m.floor_), na = (P)1 / sqrt(acc[kMom + 1] + m.floor_);
  if (lane == 0) {
#pragma unroll
    for (int k = 0; k < kMom; ++k) w[k] = acc[k] * (k < 8 ? ns : na);
    w[kW_MS] = acc[kMom];
    w[kW_MS + 1] = acc[kMom + 1];
  }
  __syncwarp();
  align_and_probe(m, w, lane);
  const int tt = (ti >= 0 && ti < m.T) ? ti : 0;
  for (int o = lane; o < kC8Dim; o += 32) {
    const P v = c8_output(m, w, o, tt);
    desc[(size_t)i * kC8Dim + o] = (v - __ldg(m.mean + o)) * __ldg(m.istd + o);
  }
  for (int k = lane; k < kC8State; k += 32) state[(size_t)i * kC8State + k] = k < kMom ? w[k] : (k == kMom ? ns : na);
}

// ---------------------------------------------------------------- node readout VJP
// Per-warp workspace of the backward: the forward's (moments, aligned,
// probes) plus the output cotangents and their images on probes, aligned
// values and moments.
constexpr int kB_G = 96;     // dE/d(raw output) [70]
constexpr int kB_DP = 166;   // probe cotangents [22] (degree one [3][4], degree two [5][2])
constexpr int kB_DA = 188;   // aligned cotangents [32]
constexpr int kB_NS = 220;   // normalizers
constexpr int kB_SIZE = 224;

template <typename P>
__device__ __forceinline__ void outer_add(P (&M)[3][3], P g, const P (&a)[3], const P (&b)[3]) {
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) M[r][c] += g * a[r] * b[c];
}

// graph_compress_kernel.cuh:909-1458: dE/d(stored descriptor) -> cotangents of
// the 40 raw moments and of the two envelope masses.
template <typename P>
__global__ void __launch_bounds__(kC8Warps * 32)
    k_c8_node_backward(C8Dev d, int nloc, const P* __restrict__ state, const P* __restrict__ dD, P* __restrict__ q) {
  __shared__ P ws[kC8Warps][kB_SIZE];
  const C8V<P> m(d);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kC8Warps + warp;
  if (i >= nloc) return;
  const P s2 = (P)1.4142135623730950488, s3 = (P)1.7320508075688772935, is5 = (P)0.44721359549995793928;
  P* w = ws[warp];
  for (int k = lane; k < kC8State; k += 32) {
    const P v = state[(size_t)i * kC8State + k];
    if (k < kMom)
      w[k] = v;
    else
      w[kB_NS + (k - kMom)] = v;
  }
  for (int k = lane; k < kC8Dim; k += 32) w[kB_G + k] = dD[(size_t)i * kC8Dim + k] * __ldg(m.istd + k);
  __syncwarp();
  align_and_probe(m, w, lane);
  const P* g = w + kB_G;
  if (lane < 4) {  // degree-one probe k = lane
    const int k = lane;
    P vk[3], d[3] = {0, 0, 0};
    probe_vec(w, k, vk);
    for (int out = 0; out < 20; ++out) {  // bispectrum 112
      const int t = out & 1;
      int a, b;
      upper_pair(out >> 1, 4, a, b);
      if (a != k && b != k) continue;
      P Q[3][3], vo[3], qo[3];
      probe_stf(w, t, Q);
      probe_vec(w, a == k ? b : a, vo);
      mat_vec(Q, vo, qo);
      const P gg = g[28 + out] * (a == b ? (P)2 : s2) * (-is5);
#pragma unroll
      for (int c = 0; c < 3; ++c) d[c] += gg * qo[c];
    }
#pragma unroll
    for (int t = 0; t < 2; ++t) {  // quartic |Q_t v_k|^2
      P Q[3][3], qv[3], qqv[3];
      probe_stf(w, t, Q);
      mat_vec(Q, vk, qv);
      mat_vec(Q, qv, qqv);
      const P gg = (P)2 * g[52 + t * 4 + k];
#pragma unroll
      for (int c = 0; c < 3; ++c) d[c] += gg * qqv[c];
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) w[kB_DP + c * 4 + k] = d[c];
  } else if (lane == 8 || lane == 9) {  // degree-two probe t
    const int t = lane - 8;
    P M[3][3] = {};
    {  // bispectrum 222: k * {tr Q0^3, s3 tr Q0^2 Q1, s3 tr Q0 Q1^2, tr Q1^3}
      P Q0[3][3], Q1[3][3], P00[3][3], P11[3][3], P01[3][3], P10[3][3];
      probe_stf(w, 0, Q0);
      probe_stf(w, 1, Q1);
      mat_mul(Q0, Q0, P00);
      mat_mul(Q1, Q1, P11);
      mat_mul(Q0, Q1, P01);
      mat_mul(Q1, Q0, P10);
      const P kb = (P)-0.58554004376911988;
      const P g0 = kb * g[48], g1 = kb * s3 * g[49], g2 = kb * s3 * g[50], g3 = kb * g[51];
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int c = 0; c < 3; ++c)
          M[r][c] = t == 0 ? (P)3 * g0 * P00[r][c] + g1 * (P01[r][c] + P10[r][c]) + g2 * P11[r][c]
                           : g1 * P00[r][c] + g2 * (P01[r][c] + P10[r][c]) + (P)3 * g3 * P11[r][c];
    }
    for (int out = t; out < 20; out += 2) {  // bispectrum 112 with tensor index t
      int a, b;
      upper_pair(out >> 1, 4, a, b);
      P va[3], vb[3];
      probe_vec(w, a, va);
      probe_vec(w, b, vb);
      outer_add(M, g[28 + out] * (a == b ? (P)1 : s2) * (-is5), va, vb);
    }
    {
      P Q[3][3];
      probe_stf(w, t, Q);
      for (int k = 0; k < 4; ++k) {  // quartic: d|Q v|^2 / dQ = 2 (Q v) v^T
        P v[3], qv[3];
        probe_vec(w, k, v);
        mat_vec(Q, v, qv);
        outer_add(M, (P)2 * g[52 + t * 4 + k], qv, v);
      }
    }
    P pg[5];
    stf_grad(M, pg);
#pragma unroll
    for (int c = 0; c < 5; ++c) w[kB_DP + 12 + c * 2 + t] = pg[c];
  }
  __syncwarp();
  {  // aligned cotangents: Gram terms plus the probe projection's transpose
    P v = 0;
    if (lane < 12) {
      const int comp = lane >> 2, ch = lane & 3;
#pragma unroll
      for (int o = 0; o < 4; ++o)
        v += (ch == o ? (P)2 : s2) * g[8 + pair_pos(ch, o, 4)] * w[kW_AV + comp * 4 + o];
#pragma unroll
      for (int k = 0; k < 4; ++k) v += m.R(4, ch, k) * w[kB_DP + comp * 4 + k];
    } else {
      const int l2 = lane - 12, comp = l2 >> 2, ch = l2 & 3;
#pragma unroll
      for (int o = 0; o < 4; ++o)
        v += (ch == o ? (P)2 : s2) * g[18 + pair_pos(ch, o, 4)] * w[kW_AT + comp * 4 + o];
#pragma unroll
      for (int k = 0; k < 2; ++k) v += m.R(6, ch, k) * w[kB_DP + 12 + comp * 2 + k];
    }
    w[kB_DA + lane] = v;
  }
  __syncwarp();
  const P ns = w[kB_NS], na = w[kB_NS + 1];
  P dm[2] = {0, 0}, sdot = 0, adot = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = lane + 32 * h;
    if (k >= kMom) continue;
    P v = 0;
    if (k < 8) {
      v = g[k];
    } else if (k < kTen) {
      const int comp = (k - kVec) >> 2, in = (k - kVec) & 3;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) v += w[kB_DA + comp * 4 + ch] * m.R(0, in, ch);
    } else {
      const int comp = (k - kTen) >> 2, in = (k - kTen) & 3;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) v += w[kB_DA + 12 + comp * 4 + ch] * m.R(2, in, ch);
    }
    dm[h] = v;
    if (k < 8)
      sdot += v * w[k];
    else
      adot += v * w[k];
  }
  sdot = wsum(sdot);
  adot = wsum(adot);
  P* qo = q + (size_t)i * kC8State;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int k = lane + 32 * h;
    if (k < kMom) qo[k] = dm[h] * (k < 8 ? ns : na);
  }
  if (lane == 0) {
    qo[kMom] = (P)0.5 * ns * (g[60] - sdot * ns);
    qo[kMom + 1] = (P)0.5 * na * (g[61] - adot * na);
  }
}

// ---------------------------------------------------------------- edge recomputation
// graph_compress_kernel.cuh:1460-1917 and the basis VJP
// (graph_compress.cuh:711-735): dE/d(r_ij) of every kept slot from the
// centre's moment cotangents, written in fp64 for the assembly.
template <typename P>
__global__ void __launch_bounds__(kC8Warps * 32)
    k_c8_edge_backward(C8Dev d, int nloc, int selt, const int* __restrict__ nl_j, const double* __restrict__ rij,
                       const int* __restrict__ atype, const P* __restrict__ qbuf, double* __restrict__ gslot) {
  const C8V<P> m(d);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i = blockIdx.x * kC8Warps + warp;
  if (i >= nloc) return;
  const int ti = atype[i];
  if (ti < 0 || ti >= m.T) return;
  P q[kC8State];
#pragma unroll
  for (int k = 0; k < kC8State; ++k) q[k] = qbuf[(size_t)i * kC8State + k];
  const P s3 = (P)1.7320508075688772935;
  const size_t row = (size_t)i * selt;
  for (int s = lane; s < selt; s += 32) {
    const int j = nl_j[row + s];
    if (j < 0) continue;
    const Geo<P> geo = c8_geometry(m, rij + 3 * (row + s));
    const P* film = m.film + ((size_t)ti * m.T + atype[j]) * 16;
    const P* trow = m.table + (size_t)geo.idx * 48;
    P rg = 0, eg = 0, db[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
    const P e2 = geo.env * geo.env;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      P k[6];
      table_coeffs(trow, c, k);
      const P fs = __ldg(film + 2 * c);
      const P fv = fs * poly(k, geo.x) + __ldg(film + 2 * c + 1), fd = fs * dpoly(k, geo.x);
      P ang = 0;
      if (c < 4) {
#pragma unroll
        for (int a = 0; a < 3; ++a) ang += q[kVec + a * 4 + c] * geo.b[1 + a];
#pragma unroll
        for (int a = 0; a < 5; ++a) ang += q[kTen + a * 4 + c] * geo.b[4 + a];
      }
      const P scaled = geo.env * ang, fg = q[c] + scaled;
      rg += geo.env * fg * fd;
      eg += (fg + scaled) * fv;
      if (c < 4) {
        const P payload = fv * e2;
#pragma unroll
        for (int a = 0; a < 3; ++a) db[1 + a] += q[kVec + a * 4 + c] * payload;
#pragma unroll
        for (int a = 0; a < 5; ++a) db[4 + a] += q[kTen + a * 4 + c] * payload;
      }
    }
    eg += (P)2 * geo.env * q[kMom] + (P)4 * e2 * geo.env * q[kMom + 1];
    rg += eg * geo.denv;
    const P ux = geo.u[0], uy = geo.u[1], uz = geo.u[2];
    const P dux = db[1] + s3 * (db[4] * uy + db[7] * uz + db[8] * ux);
    const P duy = db[2] + s3 * (db[4] * ux + db[5] * uz - db[8] * uy);
    const P duz = db[3] + s3 * (db[5] * uy + db[7] * ux) + (P)3 * db[6] * uz;
    const P dot = ux * dux + uy * duy + uz * duz;
    double* go = gslot + 3 * (row + s);
    go[0] = (double)((dux - ux * dot) * geo.iR + rg * ux);
    go[1] = (double)((duy - uy * dot) * geo.iR + rg * uy);
    go[2] = (double)((duz - uz * dot) * geo.iR + rg * uz);
  }
}

// ---------------------------------------------------------------- fitting
// components/deepmd-op/overlays/op/pt/graph_fitting.cu:1-256: one MLP shared
// by every type, h_l = act(h_{l-1} W_l + b_l) (+ h_{l-1} for a square layer
// marked residual), e = h w_head + b_head + bias_atom_e[t], and the backward
// with the seed dE/dh = w_head.  act: 0 tanh, 1 SiLU z sigmoid(z).
template <typename P>
__device__ __forceinline__ P act_v(int a, P z) {
  if (a == 0) return tanh(z);
  return z / ((P)1 + exp(-z));
}
template <typename P>
__device__ __forceinline__ P act_d(int a, P z) {
  if (a == 0) {
    const P t = tanh(z);
    return (P)1 - t * t;
  }
  const P s = (P)1 / ((P)1 + exp(-z));
  return s * ((P)1 + z * ((P)1 - s));
}

template <typename P>
struct EpiC8Fwd {
  const P* b;
  const P* X;  // residual source (the layer input), or null
  P* Z;        // pre-activation (z + b), kept for the backward
  P* Y;
  int ld, act;
  __device__ void operator()(int r, int n, P acc) const {
    const size_t o = (size_t)r * ld + n;
    const P z = acc + b[n];
    Z[o] = z;
    const P h = act_v(act, z);
    Y[o] = X ? X[o] + h : h;
  }
};

template <typename P>
struct EpiC8Bwd {
  const P* dy_next;  // residual cotangent of this layer's output, or null
  P* dX;             // cotangent of the layer input
  const P* Zprev;    // pre-activation of the previous layer, or null at the descriptor
  P* dZprev;
  int ld, act;
  __device__ void operator()(int r, int n, P acc) const {
    const size_t o = (size_t)r * ld + n;
    const P v = dy_next ? acc + dy_next[o] : acc;
    dX[o] = v;
    if (Zprev) dZprev[o] = v * act_d(act, Zprev[o]);
  }
};

// Head energy (fixed-order warp sum) and the backward seed of the last layer:
// dH = w_head, dZ = w_head * act'(Z).
template <typename P>
__global__ void k_c8_head(int nloc, int width, int act, const P* __restrict__ H, const P* __restrict__ Z,
                          const P* __restrict__ w_head, double b_head, const double* __restrict__ bias,
                          const int* __restrict__ atype, int ntypes, P* __restrict__ dH, P* __restrict__ dZ,
                          double* __restrict__ atom_e) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= nloc) return;
  const size_t r = (size_t)warp * width;
  P acc = 0;
  for (int n = lane; n < width; n += 32) {
    const P wv = __ldg(w_head + n);
    acc += H[r + n] * wv;
    dH[r + n] = wv;
    dZ[r + n] = wv * act_d(act, Z[r + n]);
  }
  acc = wsum(acc);
  if (lane == 0) {
    const int t = atype[warp];
    atom_e[warp] = (double)acc + b_head + ((t >= 0 && t < ntypes) ? bias[t] : 0.0);
  }
}

// Fused fitting (fp32): one persistent block per SM holds every weight in
// shared memory and runs forward, head and backward for 32-row tiles with the
// activations on chip.  Activations are K-major [k][row] with a row stride of
// 36 floats (float4-aligned: each warp's 4 rows arrive in one broadcast
// load); weights keep W[k][c] with an odd row stride so that both the forward
// (lanes over c) and the transposed backward (lanes over k) read distinct
// banks.  Warp w owns rows 4w..4w+3 of a tile, lane l output columns
// l, l + 32, ... ; sums run over k in order, so results do not depend on the
// launch shape.
constexpr int kFT = 32;      // rows per tile
constexpr int kFLD = 36;     // activation row stride
constexpr int kFMaxW = 128;  // widest layer the fused kernel takes

struct FusedFit {
  int L, din0, width;
  int din[kC8MaxFit], dout[kC8MaxFit], res[kC8MaxFit], ws[kC8MaxFit];
  int w_off[kC8MaxFit], b_off[kC8MaxFit];
  int wh_off, x_off, z_off[kC8MaxFit], h_off[2], dz_off[2];
  int total;  // floats of shared memory
};

FusedFit fused_fit_layout(const C8Dev& m) {
  FusedFit f{};
  f.L = m.nfit;
  f.din0 = kC8Dim;
  int o = 0, maxw = 1;
  for (int l = 0; l < f.L; ++l) {
    f.din[l] = m.fdin[l];
    f.dout[l] = m.fdout[l];
    f.res[l] = m.fres[l] && m.fdin[l] == m.fdout[l];
    f.ws[l] = m.fdout[l] | 1;
    f.w_off[l] = o;
    o += (f.din[l] * f.ws[l] + 3) / 4 * 4;  // every region starts 16-byte aligned
    f.b_off[l] = o;
    o += (f.dout[l] + 3) / 4 * 4;
    maxw = std::max(maxw, m.fdout[l]);
  }
  f.width = m.fdout[f.L - 1];
  f.wh_off = o;
  o += (f.width + 3) / 4 * 4;
  f.x_off = o;
  o += kC8Dim * kFLD;
  for (int l = 0; l < f.L; ++l) {
    f.z_off[l] = o;
    o += f.dout[l] * kFLD;
  }
  for (int k = 0; k < 2; ++k) {
    f.h_off[k] = o;
    o += maxw * kFLD;
  }
  for (int k = 0; k < 2; ++k) {
    f.dz_off[k] = o;
    o += maxw * kFLD;
  }
  f.total = o;
  return f;
}

// out[c][r] (c < N) = sum_k A[k][r] W(k, c), A K-major (ld kFLD), W(k, c) =
// T ? W[c * ws + k] : W[k * ws + c]; the epilogue sees (row, column, sum).
template <bool T, class Epi>
__device__ __forceinline__ void fit_tile_gemm(const float* A, int K, const float* W, int ws, int N, int warp,
                                              int lane, Epi epi) {
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  const int nj = (N + 31) >> 5;
  for (int k = 0; k < K; ++k) {
    const float4 a = *reinterpret_cast<const float4*>(A + k * kFLD + 4 * warp);
    float b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = lane + 32 * j;
      b[j] = (j < nj && c < N) ? (T ? W[c * ws + k] : W[k * ws + c]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[0][j] = fmaf(a.x, b[j], acc[0][j]);
      acc[1][j] = fmaf(a.y, b[j], acc[1][j]);
      acc[2][j] = fmaf(a.z, b[j], acc[2][j]);
      acc[3][j] = fmaf(a.w, b[j], acc[3][j]);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = lane + 32 * j;
    if (j < nj && c < N) {
#pragma unroll
      for (int i = 0; i < 4; ++i) epi(4 * warp + i, c, acc[i][j]);
    }
  }
}

__global__ void __launch_bounds__(256, 1)
    k_c8_fit_fused(C8Dev m, FusedFit F, int n, const int* __restrict__ atype, const float* __restrict__ desc,
                   float* __restrict__ dD, double* __restrict__ atom_e) {
  extern __shared__ __align__(16) float fs[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int act = m.act;
  for (int l = 0; l < F.L; ++l) {
    const float* w = static_cast<const float*>(m.fw[l]);
    const float* b = static_cast<const float*>(m.fb[l]);
    for (int idx = tid; idx < F.din[l] * F.dout[l]; idx += blockDim.x) {
      const int k = idx / F.dout[l], c = idx - k * F.dout[l];
      fs[F.w_off[l] + k * F.ws[l] + c] = w[idx];
    }
    for (int c = tid; c < F.dout[l]; c += blockDim.x) fs[F.b_off[l] + c] = b[c];
  }
  for (int c = tid; c < F.width; c += blockDim.x) fs[F.wh_off + c] = static_cast<const float*>(m.w_head)[c];
  __syncthreads();
  float* X = fs + F.x_off;
  const int ntiles = (n + kFT - 1) / kFT;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int r0 = tile * kFT, rows = min(kFT, n - r0);
    for (int idx = tid; idx < kFT * kC8Dim; idx += blockDim.x) {
      const int r = idx / kC8Dim, k = idx - r * kC8Dim;
      X[k * kFLD + r] = r < rows ? desc[(size_t)(r0 + r) * kC8Dim + k] : 0.f;
    }
    __syncthreads();
    // forward
    const float* in = X;
    int K = kC8Dim, hb = 0;
    for (int l = 0; l < F.L; ++l) {
      float* Z = fs + F.z_off[l];
      float* H = fs + F.h_off[hb];
      const float* bias = fs + F.b_off[l];
      const bool res = F.res[l];
      fit_tile_gemm<false>(in, K, fs + F.w_off[l], F.ws[l], F.dout[l], warp, lane, [&](int r, int c, float s) {
        const float z = s + bias[c];
        Z[c * kFLD + r] = z;
        const float h = act_v(act, z);
        H[c * kFLD + r] = res ? in[c * kFLD + r] + h : h;
      });
      __syncthreads();
      in = H;
      K = F.dout[l];
      hb ^= 1;
    }
    // head (8 lanes per row, fixed-order reduction) and the backward seed
    {
      const float* H = in;
      const float* wh = fs + F.wh_off;
      const int r = 4 * warp + (lane >> 3);
      float e = 0.f;
      for (int c = lane & 7; c < F.width; c += 8) e = fmaf(H[c * kFLD + r], wh[c], e);
      e += __shfl_xor_sync(0xffffffffu, e, 1);
      e += __shfl_xor_sync(0xffffffffu, e, 2);
      e += __shfl_xor_sync(0xffffffffu, e, 4);
      if ((lane & 7) == 0 && r < rows) {
        const int t = atype[r0 + r];
        atom_e[r0 + r] = (double)e + m.b_head + ((t >= 0 && t < m.ntypes) ? m.bias[t] : 0.0);
      }
    }
    __syncthreads();  // the last H is dead: its buffer and the other one now carry dH
    float* dH = fs + F.h_off[0];
    float* dZ = fs + F.dz_off[0];
    {
      const float* Zl = fs + F.z_off[F.L - 1];
      const float* wh = fs + F.wh_off;
      for (int idx = tid; idx < F.width * kFT; idx += blockDim.x) {
        const int c = idx / kFT, r = idx - c * kFT;
        dH[c * kFLD + r] = wh[c];
        dZ[c * kFLD + r] = wh[c] * act_d(act, Zl[c * kFLD + r]);
      }
    }
    __syncthreads();
    int cur = 0;
    for (int l = F.L - 1; l >= 0; --l) {
      const float* dZc = fs + F.dz_off[cur];
      const float* dHc = fs + F.h_off[cur];
      float* dZn = fs + F.dz_off[cur ^ 1];
      float* dHn = fs + F.h_off[cur ^ 1];
      const float* Zp = l > 0 ? fs + F.z_off[l - 1] : nullptr;
      const bool res = F.res[l];
      fit_tile_gemm<true>(dZc, F.dout[l], fs + F.w_off[l], F.ws[l], F.din[l], warp, lane, [&](int r, int c, float s) {
        const float v = res ? s + dHc[c * kFLD + r] : s;
        if (Zp) {
          dHn[c * kFLD + r] = v;
          dZn[c * kFLD + r] = v * act_d(act, Zp[c * kFLD + r]);
        } else if (r < rows) {
          dD[(size_t)(r0 + r) * kC8Dim + c] = v;
        }
      });
      __syncthreads();
      cur ^= 1;
    }
  }
}

bool fused_fit_ok(const C8Dev& m, const FusedFit& F) {
  if (m.nfit < 1 || m.nfit > kC8MaxFit) return false;
  for (int l = 0; l < m.nfit; ++l)
    if (m.fdin[l] > kFMaxW || m.fdout[l] > kFMaxW) return false;
  return (size_t)F.total * sizeof(float) <= 220 * 1024;
}

}  // namespace

template <typename P>
void launch_c8_forward(cudaStream_t st, const C8Dev& m, int nloc, int selt, const int* nl_j, const double* rij,
                       const int* atype, const C8Work<P>& w) {
  if (nloc <= 0) return;
  count_launch();
  k_c8_forward<P><<<(nloc + kC8Warps - 1) / kC8Warps, kC8Warps * 32, 0, st>>>(m, nloc, selt, nl_j, rij, atype,
                                                                               w.desc, w.state);
}

template <typename P>
void launch_c8_fitting(cudaStream_t st, const C8Dev& m, int nloc, const int* atype, const C8Work<P>& w,
                       double* atom_e) {
  if (nloc <= 0) return;
  if constexpr (std::is_same<P, float>::value) {
    const FusedFit F = fused_fit_layout(m);
    if (fused_fit_ok(m, F)) {
      static int nsm = 0;
      const size_t smem = (size_t)F.total * sizeof(float);
      static size_t attr = 0;
      if (!nsm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
      }
      if (smem > attr) {
        cudaFuncSetAttribute(k_c8_fit_fused, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr = smem;
      }
      const int ntiles = (nloc + kFT - 1) / kFT;
      count_launch();
      k_c8_fit_fused<<<std::min(ntiles, std::max(nsm, 1)), 256, smem, st>>>(m, F, nloc, atype, w.desc, w.dD, atom_e);
      return;
    }
  }
  const int L = m.nfit;
  const P* X = w.desc;
  for (int l = 0; l < L; ++l) {
    const int din = m.fdin[l], dout = m.fdout[l];
    EpiC8Fwd<P> epi{static_cast<const P*>(m.fb[l]), (m.fres[l] && din == dout) ? X : nullptr, w.Z[l], w.H[l],
                    dout, m.act};
    dim3 grid((dout + kBN - 1) / kBN, (nloc + kBM - 1) / kBM);
    count_launch();
    k_gemm<P, false, EpiC8Fwd<P>><<<grid, 256, 0, st>>>(nullptr, dout, din, X, din, static_cast<const P*>(m.fw[l]),
                                                        dout, epi, nloc);
    X = w.H[l];
  }
  const int width = m.fdout[L - 1];
  count_launch();
  k_c8_head<P><<<(nloc * 32 + 255) / 256, 256, 0, st>>>(nloc, width, m.act, w.H[L - 1], w.Z[L - 1],
                                                        static_cast<const P*>(m.w_head), m.b_head, m.bias, atype,
                                                        m.ntypes, w.dH[0], w.dZ[0], atom_e);
  // backward: dZ_l (cur) -> dX = dZ_l W_l^T (+ dH_l when residual) -> dZ_{l-1}
  int cur = 0;
  for (int l = L - 1; l >= 0; --l) {
    const int din = m.fdin[l], dout = m.fdout[l];
    const bool res = m.fres[l] && din == dout;
    P* dX = l > 0 ? w.dH[cur ^ 1] : w.dD;
    EpiC8Bwd<P> epi{res ? w.dH[cur] : nullptr, dX, l > 0 ? w.Z[l - 1] : nullptr, l > 0 ? w.dZ[cur ^ 1] : nullptr,
                    din, m.act};
    dim3 grid((din + kBN - 1) / kBN, (nloc + kBM - 1) / kBM);
    count_launch();
    k_gemm<P, true, EpiC8Bwd<P>><<<grid, 256, 0, st>>>(nullptr, din, dout, w.dZ[cur], dout,
                                                       static_cast<const P*>(m.fw[l]), dout, epi, nloc);
    cur ^= 1;
  }
}

template <typename P>
void launch_c8_node_backward(cudaStream_t st, const C8Dev& m, int nloc, const C8Work<P>& w) {
  if (nloc <= 0) return;
  count_launch();
  k_c8_node_backward<P><<<(nloc + kC8Warps - 1) / kC8Warps, kC8Warps * 32, 0, st>>>(m, nloc, w.state, w.dD, w.q);
}

template <typename P>
void launch_c8_edge_backward(cudaStream_t st, const C8Dev& m, int nloc, int selt, const int* nl_j,
                             const double* rij, const int* atype, const C8Work<P>& w, double* gslot) {
  if (nloc <= 0) return;
  count_launch();
  k_c8_edge_backward<P><<<(nloc + kC8Warps - 1) / kC8Warps, kC8Warps * 32, 0, st>>>(m, nloc, selt, nl_j, rij,
                                                                                    atype, w.q, gslot);
}

#define B200DP_C8_INST(P)                                                                                        \
  template void launch_c8_forward<P>(cudaStream_t, const C8Dev&, int, int, const int*, const double*, const int*, \
                                     const C8Work<P>&);                                                          \
  template void launch_c8_fitting<P>(cudaStream_t, const C8Dev&, int, const int*, const C8Work<P>&, double*);     \
  template void launch_c8_node_backward<P>(cudaStream_t, const C8Dev&, int, const C8Work<P>&);                   \
  template void launch_c8_edge_backward<P>(cudaStream_t, const C8Dev&, int, int, const int*, const double*,      \
                                           const int*, const C8Work<P>&, double*);

B200DP_C8_INST(float)
B200DP_C8_INST(double)

}  // namespace b200dp
