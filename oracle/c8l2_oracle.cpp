// CPU oracle of the C8L2 profile (test infrastructure only: used by tests/,
// __graft_entry__.smoke() and bench.py's CPU-baseline leg, never by the
// product path).
//
// A plain fp64 restatement of the reference's compressed degree-wise DPA4C
// descriptor with Channels = 8, Lmax = 2, no radial modes and no spin, its
// fitting net, the node-readout VJP and the edge recomputation that gives
// dE/d(edge vector), then the dual-CSR force / virial assembly.  Each step
// cites the reference text it restates (paths inside the dpa4c-runtime
// project):
//
//   geometry, envelope     include/dpa_chain/graph_compress.cuh:218-266
//   radial table           include/dpa_chain/graph_compress.cuh:97-154
//   angular basis l <= 2   include/dpa_chain/graph_compress.cuh:292-304
//   STF algebra            include/dpa_chain/graph_compress.cuh:565-626
//   widths and layout      include/dpa_chain/graph_compress_launch.h:270-396
//   forward steps 1-5      components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh:130-710
//   fitting                components/deepmd-op/overlays/op/pt/graph_fitting.cu:1-256
//   node VJP               components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh:769-1458
//   edge backward          components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh:1460-1917
//   basis VJP              include/dpa_chain/graph_compress.cuh:711-735
//   force / virial         components/deepmd-op/overlays/op/pt/edge_force_virial.cu:1-14
//
// Parity status: pinned to the reference source text, and to outputs of the
// reference's own descriptor kernels run on a B200 (golden fixtures under
// tests/golden/, made by tests/golden/make_c8l2_golden.py with the harness in
// oracle/ref_c8l2.cu).  The edge list is this framework's formatted
// neighbour list (kept slots of every centre row).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

namespace {

constexpr int C0 = 8, C1 = 4, C2 = 4, K1 = 4, K2 = 2;
constexpr int VEC = C0, TEN = C0 + 3 * C1, MW = TEN + 5 * C2;  // 40 moments
constexpr int SW = MW + 2;                                     // + 2 norms
constexpr int OG1 = C0, OG2 = OG1 + 10, OB112 = OG2 + 10, OB222 = OB112 + 20, OQ = OB222 + 4, ODIV = OQ + 8,
              OTYPE = ODIV + 2, DW = OTYPE + C0;  // 70
static_assert(DW == 70, "C8L2 descriptor width");

const double kS2 = std::sqrt(2.0), kS3 = std::sqrt(3.0), kIS2 = 1.0 / std::sqrt(2.0), kIS5 = 1.0 / std::sqrt(5.0),
             kIS6 = 1.0 / std::sqrt(6.0);
constexpr double kBis222 = -0.58554004376911988;

struct FitLayer {
  int din, dout;
  std::vector<double> w, b;
};

struct C8 {
  int T = 0, nint = 0, act = 1;
  std::vector<int> fit, res, sel;
  double stride = 0, tmax = 0, rcut = 0, eps = 0, floor_ = 0, b_head = 0;
  std::vector<double> bias, table, film, temb, readout, mean, istd, w_head;
  std::vector<FitLayer> layers;
};

std::string g_err;

bool load(const char* path, C8& m) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    g_err = "cannot open model";
    return false;
  }
  std::vector<char> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  size_t off = 0;
  bool bad = false;
  auto rd = [&](void* d, size_t n) {
    if (off + n > buf.size()) {
      bad = true;
      std::memset(d, 0, n);
    } else {
      std::memcpy(d, buf.data() + off, n);
    }
    off += n;
  };
  auto ri = [&]() {
    int32_t v;
    rd(&v, 4);
    return (int)v;
  };
  auto rv = [&](std::vector<double>& v, size_t n) {
    v.resize(n);
    rd(v.data(), 8 * n);
  };
  if (buf.size() < 8 || std::memcmp(buf.data(), "B2DPC8L2", 8) != 0) {
    g_err = "bad magic";
    return false;
  }
  off = 8;
  if (ri() != 1) {
    g_err = "bad version";
    return false;
  }
  m.T = ri();
  const int ch = ri(), lmax = ri();
  m.nint = ri();
  const int width = ri(), nf = ri();
  if (m.T <= 0 || m.T > 8 || ch != C0 || lmax != 2 || width != C0 || nf < 1 || nf > 8 || m.nint <= 0) {
    g_err = "unsupported C8L2 header";
    return false;
  }
  for (int i = 0; i < nf; ++i) m.fit.push_back(ri());
  for (int i = 0; i < nf; ++i) m.res.push_back(ri());
  m.act = ri();
  for (int t = 0; t < m.T; ++t) m.sel.push_back(ri());
  double d[6];
  rd(d, sizeof(d));
  m.stride = d[0], m.tmax = d[1], m.rcut = d[2], m.eps = d[3], m.floor_ = d[4], m.b_head = d[5];
  rv(m.bias, m.T);
  rv(m.table, (size_t)m.nint * 6 * C0);
  rv(m.film, (size_t)m.T * m.T * C0 * 2);
  rv(m.temb, (size_t)m.T * C0);
  rv(m.readout, 8 * 16);
  rv(m.mean, DW);
  rv(m.istd, DW);
  int din = DW;
  for (int l = 0; l < nf; ++l) {
    FitLayer L;
    L.din = din;
    L.dout = m.fit[l];
    rv(L.w, (size_t)din * L.dout);
    rv(L.b, L.dout);
    m.layers.push_back(std::move(L));
    din = m.fit[l];
  }
  rv(m.w_head, din);
  if (bad || off != buf.size()) {
    g_err = "truncated or oversized model file";
    return false;
  }
  return true;
}

// Readout matrix k (4 x 4 storage), entry [row][column].
inline double ro(const C8& m, int k, int r, int c) { return m.readout[(size_t)k * 16 + r * 4 + c]; }

// graph_compress.cuh:218-226
double envelope(double r, double rc) {
  const double u = std::fmin(std::fmax((rc - r) / rc, 0.0), 1.0), x = 1.0 - u;
  const double s = 1.0 + x * (4.0 + x * (10.0 + x * (20.0 + 35.0 * x)));
  return u * u * u * u * s;
}
// graph_compress.cuh:228-243
double envelope_derivative(double r, double rc) {
  if (r <= 0.0 || r >= rc) return 0.0;
  const double x = r / rc, u = 1.0 - x;
  const double s = 1.0 + 4.0 * x + 10.0 * x * x + 20.0 * x * x * x + 35.0 * x * x * x * x;
  const double ds = 4.0 + 20.0 * x + 60.0 * x * x + 140.0 * x * x * x;
  return (-4.0 * u * u * u * s + u * u * u * u * ds) / rc;
}

struct Geo {
  double u[3], R, iR, env, denv;
  double basis[9];
  int idx;
  double x;
};

// Regularized distance, unit direction, envelope and l <= 2 harmonics
// (graph_compress.cuh:250-266, 292-304); canonical table location
// (graph_compress.cuh:97-106: no clamping, last interval extrapolates).
Geo geometry(const C8& m, const double* r) {
  Geo g;
  const double sq = r[0] * r[0] + r[1] * r[1] + r[2] * r[2] + m.eps * m.eps;
  g.R = std::sqrt(sq);
  g.iR = 1.0 / g.R;
  for (int c = 0; c < 3; ++c) g.u[c] = r[c] * g.iR;
  g.env = envelope(g.R, m.rcut);
  g.denv = envelope_derivative(g.R, m.rcut);
  const double x = g.u[0], y = g.u[1], z = g.u[2];
  g.basis[0] = 1.0;
  g.basis[1] = x;
  g.basis[2] = y;
  g.basis[3] = z;
  g.basis[4] = kS3 * x * y;
  g.basis[5] = kS3 * y * z;
  g.basis[6] = 0.5 * (3.0 * z * z - 1.0);
  g.basis[7] = kS3 * x * z;
  g.basis[8] = 0.5 * kS3 * (x * x - y * y);
  int idx = (int)(g.R / m.stride);
  if (idx > m.nint - 1) idx = m.nint - 1;
  g.idx = idx;
  g.x = g.R - idx * m.stride;
  return g;
}

// Channel c of the quintic table and its derivative (graph_compress.cuh:127-154).
void radial(const C8& m, const Geo& g, int c, double& v, double& dv) {
  const double* row = m.table.data() + (size_t)g.idx * 6 * C0;
  const double* q = row + 4 * c;
  const double* p = row + 4 * C0 + 2 * c;
  const double x = g.x;
  v = q[0] + (q[1] + (q[2] + (q[3] + (p[0] + p[1] * x) * x) * x) * x) * x;
  dv = q[1] + (2.0 * q[2] + (3.0 * q[3] + (4.0 * p[0] + 5.0 * p[1] * x) * x) * x) * x;
}

// packed_to_stf (graph_compress.cuh:567-577)
void stf(const double* p, double M[3][3]) {
  M[0][0] = -p[2] * kIS6 + p[4] * kIS2;
  M[1][1] = -p[2] * kIS6 - p[4] * kIS2;
  M[2][2] = 2.0 * p[2] * kIS6;
  M[0][1] = M[1][0] = p[0] * kIS2;
  M[1][2] = M[2][1] = p[1] * kIS2;
  M[0][2] = M[2][0] = p[3] * kIS2;
}
// matrix_gradient_to_packed (graph_compress.cuh:612-621)
void stf_grad(const double M[3][3], double* g) {
  g[0] = (M[0][1] + M[1][0]) * kIS2;
  g[1] = (M[1][2] + M[2][1]) * kIS2;
  g[2] = (-M[0][0] - M[1][1] + 2.0 * M[2][2]) * kIS6;
  g[3] = (M[0][2] + M[2][0]) * kIS2;
  g[4] = (M[0][0] - M[1][1]) * kIS2;
}
void mat_mul(const double A[3][3], const double B[3][3], double C[3][3]) {
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < 3; ++j) {
      double s = 0;
      for (int k = 0; k < 3; ++k) s += A[i][k] * B[k][j];
      C[i][j] = s;
    }
}
void mat_vec(const double A[3][3], const double* v, double* o) {
  for (int i = 0; i < 3; ++i) o[i] = A[i][0] * v[0] + A[i][1] * v[1] + A[i][2] * v[2];
}

// decode_upper_pair (graph_compress.cuh:638-647)
void upper_pair(int pair, int width, int& r, int& c) {
  r = 0;
  while (pair >= width - r) {
    pair -= width - r;
    ++r;
  }
  c = r + pair;
}

struct NodeFwd {
  double m[MW];  // normalized moments
  double ns, na, ms, ma;
  double av[3][C1], at[5][C2];  // aligned
  double pv[3][K1], pt[5][K2];  // probes
  double raw_out[DW];           // invariants before the output normalization
};

// Forward steps 2-5 of one node from its raw moments and masses.
void node_forward(const C8& m, const double* raw, double ms, double ma, int type, NodeFwd& n) {
  n.ms = ms;
  n.ma = ma;
  n.ns = 1.0 / std::sqrt(ms + m.floor_);
  n.na = 1.0 / std::sqrt(ma + m.floor_);
  for (int k = 0; k < MW; ++k) n.m[k] = raw[k] * (k < C0 ? n.ns : n.na);
  for (int c = 0; c < 3; ++c)
    for (int ch = 0; ch < C1; ++ch) {
      double s = 0;
      for (int in = 0; in < C1; ++in) s += n.m[VEC + c * C1 + in] * ro(m, 0, in, ch);
      n.av[c][ch] = s;
    }
  for (int c = 0; c < 5; ++c)
    for (int ch = 0; ch < C2; ++ch) {
      double s = 0;
      for (int in = 0; in < C2; ++in) s += n.m[TEN + c * C2 + in] * ro(m, 2, in, ch);
      n.at[c][ch] = s;
    }
  for (int c = 0; c < 3; ++c)
    for (int k = 0; k < K1; ++k) {
      double s = 0;
      for (int in = 0; in < C1; ++in) s += n.av[c][in] * ro(m, 4, in, k);
      n.pv[c][k] = s;
    }
  for (int c = 0; c < 5; ++c)
    for (int k = 0; k < K2; ++k) {
      double s = 0;
      for (int in = 0; in < C2; ++in) s += n.at[c][in] * ro(m, 6, in, k);
      n.pt[c][k] = s;
    }
  double* o = n.raw_out;
  for (int c = 0; c < C0; ++c) {
    o[c] = n.m[c];
    o[OTYPE + c] = m.temb[(size_t)type * C0 + c];
  }
  for (int p = 0; p < 10; ++p) {
    int r, c;
    upper_pair(p, C1, r, c);
    double s = 0;
    for (int k = 0; k < 3; ++k) s += n.av[k][r] * n.av[k][c];
    o[OG1 + p] = (r == c ? 1.0 : kS2) * s;
    upper_pair(p, C2, r, c);
    s = 0;
    for (int k = 0; k < 5; ++k) s += n.at[k][r] * n.at[k][c];
    o[OG2 + p] = (r == c ? 1.0 : kS2) * s;
  }
  double Q[K2][3][3];
  for (int t = 0; t < K2; ++t) {
    double pk[5];
    for (int k = 0; k < 5; ++k) pk[k] = n.pt[k][t];
    stf(pk, Q[t]);
  }
  for (int out = 0; out < 20; ++out) {
    const int t = out % K2;
    int a, b;
    upper_pair(out / K2, K1, a, b);
    const double l[3] = {n.pv[0][a], n.pv[1][a], n.pv[2][a]}, rr[3] = {n.pv[0][b], n.pv[1][b], n.pv[2][b]};
    double pr[3];
    mat_vec(Q[t], rr, pr);
    o[OB112 + out] = (a == b ? 1.0 : kS2) * (-kIS5) * (l[0] * pr[0] + l[1] * pr[1] + l[2] * pr[2]);
  }
  static const int ent[4][3] = {{0, 0, 0}, {0, 0, 1}, {0, 1, 1}, {1, 1, 1}};
  const double sc[4] = {1.0, kS3, kS3, 1.0};
  for (int k = 0; k < 4; ++k) {
    double AB[3][3], ABC[3][3];
    mat_mul(Q[ent[k][0]], Q[ent[k][1]], AB);
    mat_mul(AB, Q[ent[k][2]], ABC);
    o[OB222 + k] = sc[k] * kBis222 * (ABC[0][0] + ABC[1][1] + ABC[2][2]);
  }
  for (int out = 0; out < 8; ++out) {
    const int vi = out % K1, ti = out / K1;
    const double v[3] = {n.pv[0][vi], n.pv[1][vi], n.pv[2][vi]};
    double pr[3];
    mat_vec(Q[ti], v, pr);
    o[OQ + out] = pr[0] * pr[0] + pr[1] * pr[1] + pr[2] * pr[2];
  }
  o[ODIV] = std::sqrt(ms + m.floor_);
  o[ODIV + 1] = std::sqrt(ma + m.floor_);
}

// Node VJP: dE/d(raw output) -> cotangents of the raw moments (40) and of the
// two envelope masses (graph_compress_kernel.cuh:909-1458).
void node_backward(const C8& m, const NodeFwd& n, const double* gout, double* q) {
  double dpv[3][K1] = {}, dpt[5][K2] = {}, dav[3][C1] = {}, dat[5][C2] = {}, dm[MW] = {};
  double Q[K2][3][3];
  for (int t = 0; t < K2; ++t) {
    double pk[5];
    for (int k = 0; k < 5; ++k) pk[k] = n.pt[k][t];
    stf(pk, Q[t]);
  }
  // bispectrum 112: value = cf (-1/sqrt5) a^T Q_t b
  for (int out = 0; out < 20; ++out) {
    const int t = out % K2;
    int a, b;
    upper_pair(out / K2, K1, a, b);
    const double g = gout[OB112 + out] * (a == b ? 1.0 : kS2) * (-kIS5);
    const double va[3] = {n.pv[0][a], n.pv[1][a], n.pv[2][a]}, vb[3] = {n.pv[0][b], n.pv[1][b], n.pv[2][b]};
    double Qa[3], Qb[3];
    mat_vec(Q[t], vb, Qb);
    mat_vec(Q[t], va, Qa);
    for (int c = 0; c < 3; ++c) {
      dpv[c][a] += g * Qb[c];
      dpv[c][b] += g * Qa[c];
    }
    double M[3][3];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) M[i][j] = g * va[i] * vb[j];
    double pg[5];
    stf_grad(M, pg);
    for (int c = 0; c < 5; ++c) dpt[c][t] += pg[c];
  }
  // bispectrum 222
  {
    static const int ent[4][3] = {{0, 0, 0}, {0, 0, 1}, {0, 1, 1}, {1, 1, 1}};
    const double sc[4] = {1.0, kS3, kS3, 1.0};
    double dQ[K2][3][3] = {};
    for (int k = 0; k < 4; ++k) {
      const double g = gout[OB222 + k] * sc[k] * kBis222;
      const int A = ent[k][0], B = ent[k][1], Cc = ent[k][2];
      double BC[3][3], CA[3][3], AB[3][3];
      mat_mul(Q[B], Q[Cc], BC);
      mat_mul(Q[Cc], Q[A], CA);
      mat_mul(Q[A], Q[B], AB);
      // d tr(ABC)/dA = (BC)^T, /dB = (CA)^T, /dC = (AB)^T
      for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j) {
          dQ[A][i][j] += g * BC[j][i];
          dQ[B][i][j] += g * CA[j][i];
          dQ[Cc][i][j] += g * AB[j][i];
        }
    }
    for (int t = 0; t < K2; ++t) {
      double pg[5];
      stf_grad(dQ[t], pg);
      for (int c = 0; c < 5; ++c) dpt[c][t] += pg[c];
    }
  }
  // quartic: |Q_t v|^2
  for (int out = 0; out < 8; ++out) {
    const int vi = out % K1, ti = out / K1;
    const double g = gout[OQ + out];
    const double v[3] = {n.pv[0][vi], n.pv[1][vi], n.pv[2][vi]};
    double Qv[3], QQv[3];
    mat_vec(Q[ti], v, Qv);
    mat_vec(Q[ti], Qv, QQv);
    for (int c = 0; c < 3; ++c) dpv[c][vi] += 2.0 * g * QQv[c];
    double M[3][3];
    for (int i = 0; i < 3; ++i)
      for (int j = 0; j < 3; ++j) M[i][j] = 2.0 * g * Qv[i] * v[j];
    double pg[5];
    stf_grad(M, pg);
    for (int c = 0; c < 5; ++c) dpt[c][ti] += pg[c];
  }
  // Grams
  for (int p = 0; p < 10; ++p) {
    int r, c;
    upper_pair(p, C1, r, c);
    double g = gout[OG1 + p] * (r == c ? 1.0 : kS2);
    for (int k = 0; k < 3; ++k) {
      dav[k][r] += g * n.av[k][c];
      dav[k][c] += g * n.av[k][r];
    }
    upper_pair(p, C2, r, c);
    g = gout[OG2 + p] * (r == c ? 1.0 : kS2);
    for (int k = 0; k < 5; ++k) {
      dat[k][r] += g * n.at[k][c];
      dat[k][c] += g * n.at[k][r];
    }
  }
  // probes -> aligned
  for (int c = 0; c < 3; ++c)
    for (int in = 0; in < C1; ++in) {
      double s = 0;
      for (int k = 0; k < K1; ++k) s += dpv[c][k] * ro(m, 4, in, k);
      dav[c][in] += s;
    }
  for (int c = 0; c < 5; ++c)
    for (int in = 0; in < C2; ++in) {
      double s = 0;
      for (int k = 0; k < K2; ++k) s += dpt[c][k] * ro(m, 6, in, k);
      dat[c][in] += s;
    }
  // aligned -> normalized moments
  for (int c = 0; c < C0; ++c) dm[c] = gout[c];
  for (int c = 0; c < 3; ++c)
    for (int in = 0; in < C1; ++in) {
      double s = 0;
      for (int ch = 0; ch < C1; ++ch) s += dav[c][ch] * ro(m, 0, in, ch);
      dm[VEC + c * C1 + in] = s;
    }
  for (int c = 0; c < 5; ++c)
    for (int in = 0; in < C2; ++in) {
      double s = 0;
      for (int ch = 0; ch < C2; ++ch) s += dat[c][ch] * ro(m, 2, in, ch);
      dm[TEN + c * C2 + in] = s;
    }
  double sdot = 0, adot = 0;
  for (int k = 0; k < MW; ++k) (k < C0 ? sdot : adot) += dm[k] * n.m[k];
  for (int k = 0; k < MW; ++k) q[k] = dm[k] * (k < C0 ? n.ns : n.na);
  q[MW] = 0.5 * n.ns * (gout[ODIV] - sdot * n.ns);
  q[MW + 1] = 0.5 * n.na * (gout[ODIV + 1] - adot * n.na);
}

double act(int a, double z) { return a == 0 ? std::tanh(z) : z / (1.0 + std::exp(-z)); }
double dact(int a, double z) {
  if (a == 0) {
    const double t = std::tanh(z);
    return 1.0 - t * t;
  }
  const double s = 1.0 / (1.0 + std::exp(-z));
  return s * (1.0 + z * (1.0 - s));
}

// Fitting (graph_fitting.cu:1-20, 150-256): h_l = act(h_{l-1} W_l + b_l)
// (+ h_{l-1} when the layer is square and marked residual); e = h w_head +
// b_head + bias_atom_e[t].  Returns e and dE/dx.
double fitting(const C8& m, const double* x, int type, double* dx) {
  const int L = (int)m.layers.size();
  std::vector<std::vector<double>> h(L + 1), pre(L);
  h[0].assign(x, x + DW);
  for (int l = 0; l < L; ++l) {
    const FitLayer& F = m.layers[l];
    pre[l].assign(F.dout, 0.0);
    for (int o = 0; o < F.dout; ++o) {
      double s = F.b[o];
      for (int i = 0; i < F.din; ++i) s += h[l][i] * F.w[(size_t)i * F.dout + o];
      pre[l][o] = s;
    }
    h[l + 1].resize(F.dout);
    const bool res = m.res[l] && F.din == F.dout;
    for (int o = 0; o < F.dout; ++o) h[l + 1][o] = act(m.act, pre[l][o]) + (res ? h[l][o] : 0.0);
  }
  double e = m.b_head + m.bias[type];
  for (size_t o = 0; o < m.w_head.size(); ++o) e += h[L][o] * m.w_head[o];
  std::vector<double> dh(m.w_head);
  for (int l = L - 1; l >= 0; --l) {
    const FitLayer& F = m.layers[l];
    const bool res = m.res[l] && F.din == F.dout;
    std::vector<double> dz(F.dout), dprev(F.din, 0.0);
    for (int o = 0; o < F.dout; ++o) dz[o] = dh[o] * dact(m.act, pre[l][o]);
    for (int i = 0; i < F.din; ++i) {
      double s = res ? dh[i] : 0.0;
      for (int o = 0; o < F.dout; ++o) s += dz[o] * F.w[(size_t)i * F.dout + o];
      dprev[i] = s;
    }
    dh.swap(dprev);
  }
  for (int k = 0; k < DW; ++k) dx[k] = dh[k];
  return e;
}

struct Handle {
  C8 m;
};

}  // namespace

extern "C" {

const char* c8_last_error() { return g_err.c_str(); }

void* c8_load(const char* path) {
  auto* h = new Handle;
  if (!load(path, h->m)) {
    delete h;
    return nullptr;
  }
  return h;
}

void c8_free(void* h) { delete static_cast<Handle*>(h); }

// Energy, forces (nall x 3), virial (9), per-atom energy (nloc) and per-atom
// virial (nall x 9, on the neighbour end of each edge), plus optional
// per-centre descriptor (nloc x 70, after the output normalization), state
// (nloc x 42: normalized moments, scalar and angular normalizers), dE/dD
// (nloc x 70, w.r.t. the stored descriptor) and moment cotangents q
// (nloc x 42: raw moments, then the two masses), and dE/d(edge vector) per
// slot (nloc x selt x 3, zero at empty slots).  The edges are the kept slots
// (nl_j >= 0) of the formatted list; rij[slot] = x_j - x_i.
int c8_compute(void* hp, int nloc, int nall, int selt, const int* nl_j, const double* rij, const int* atype,
               double* energy, double* force, double* virial, double* atom_e, double* atom_virial, double* descriptor,
               double* state, double* grad_descriptor, double* qout, double* edge_grad) {
  const C8& m = static_cast<Handle*>(hp)->m;
  for (int i = 0; i < nall; ++i)
    if (atype[i] < 0 || atype[i] >= m.T) {
      g_err = "bad atom type";
      return 1;
    }
  std::vector<double> g((size_t)nloc * selt * 3, 0.0), ae(nloc);
#pragma omp parallel for schedule(dynamic, 16)
  for (int i = 0; i < nloc; ++i) {
    const int ti = atype[i];
    double raw[MW] = {}, ms = 0, ma = 0;
    for (int s = 0; s < selt; ++s) {
      const size_t slot = (size_t)i * selt + s;
      const int j = nl_j[slot];
      if (j < 0) continue;
      const Geo geo = geometry(m, rij + 3 * slot);
      const double* film = m.film.data() + ((size_t)ti * m.T + atype[j]) * C0 * 2;
      for (int c = 0; c < C0; ++c) {
        double v, dv;
        radial(m, geo, c, v, dv);
        const double amp = (film[2 * c] * v + film[2 * c + 1]) * geo.env;
        const double ang = amp * geo.env;
        raw[c] += amp;
        if (c < C1)
          for (int k = 0; k < 3; ++k) raw[VEC + k * C1 + c] += ang * geo.basis[1 + k];
        if (c < C2)
          for (int k = 0; k < 5; ++k) raw[TEN + k * C2 + c] += ang * geo.basis[4 + k];
      }
      const double e2 = geo.env * geo.env;
      ms += e2;
      ma += e2 * e2;
    }
    NodeFwd n;
    node_forward(m, raw, ms, ma, ti, n);
    double d[DW], dd[DW], gout[DW], q[SW];
    for (int k = 0; k < DW; ++k) d[k] = (n.raw_out[k] - m.mean[k]) * m.istd[k];
    ae[i] = fitting(m, d, ti, dd);
    for (int k = 0; k < DW; ++k) gout[k] = dd[k] * m.istd[k];
    node_backward(m, n, gout, q);
    if (descriptor)
      for (int k = 0; k < DW; ++k) descriptor[(size_t)i * DW + k] = d[k];
    if (grad_descriptor)
      for (int k = 0; k < DW; ++k) grad_descriptor[(size_t)i * DW + k] = dd[k];
    if (state) {
      for (int k = 0; k < MW; ++k) state[(size_t)i * SW + k] = n.m[k];
      state[(size_t)i * SW + MW] = n.ns;
      state[(size_t)i * SW + MW + 1] = n.na;
    }
    if (qout)
      for (int k = 0; k < SW; ++k) qout[(size_t)i * SW + k] = q[k];
    // edge recomputation (graph_compress_kernel.cuh:1632-1830)
    for (int s = 0; s < selt; ++s) {
      const size_t slot = (size_t)i * selt + s;
      const int j = nl_j[slot];
      if (j < 0) continue;
      const Geo geo = geometry(m, rij + 3 * slot);
      const double* film = m.film.data() + ((size_t)ti * m.T + atype[j]) * C0 * 2;
      double rg = 0, eg = 0, db[9] = {};
      for (int c = 0; c < C0; ++c) {
        double v, dv;
        radial(m, geo, c, v, dv);
        const double fv = film[2 * c] * v + film[2 * c + 1], fd = film[2 * c] * dv;
        double ang = 0;
        if (c < C1)
          for (int k = 0; k < 3; ++k) ang += q[VEC + k * C1 + c] * geo.basis[1 + k];
        if (c < C2)
          for (int k = 0; k < 5; ++k) ang += q[TEN + k * C2 + c] * geo.basis[4 + k];
        const double scaled = geo.env * ang, fg = q[c] + scaled;
        rg += geo.env * fg * fd;
        eg += (fg + scaled) * fv;
        const double payload = fv * geo.env * geo.env;
        if (c < C1)
          for (int k = 0; k < 3; ++k) db[1 + k] += q[VEC + k * C1 + c] * payload;
        if (c < C2)
          for (int k = 0; k < 5; ++k) db[4 + k] += q[TEN + k * C2 + c] * payload;
      }
      const double e2 = geo.env * geo.env;
      eg += 2.0 * geo.env * q[MW] + 4.0 * e2 * geo.env * q[MW + 1];
      rg += eg * geo.denv;
      // basis_vjp (graph_compress.cuh:711-735)
      const double ux = geo.u[0], uy = geo.u[1], uz = geo.u[2];
      const double dux = db[1] + kS3 * (db[4] * uy + db[7] * uz + db[8] * ux);
      const double duy = db[2] + kS3 * (db[4] * ux + db[5] * uz - db[8] * uy);
      const double duz = db[3] + kS3 * (db[5] * uy + db[7] * ux) + 3.0 * db[6] * uz;
      const double dot = ux * dux + uy * duy + uz * duz;
      double* go = g.data() + 3 * slot;
      go[0] = (dux - ux * dot) * geo.iR + rg * ux;
      go[1] = (duy - uy * dot) * geo.iR + rg * uy;
      go[2] = (duz - uz * dot) * geo.iR + rg * uz;
    }
  }
  // assembly (edge_force_virial.cu:1-14): F[dst] += g, F[src] -= g,
  // atom_virial[src] += -g (x) r; serial, fixed order
  std::vector<double> f((size_t)nall * 3, 0.0), av((size_t)nall * 9, 0.0);
  double v[9] = {}, e = 0;
  for (int i = 0; i < nloc; ++i) {
    e += ae[i];
    for (int s = 0; s < selt; ++s) {
      const size_t slot = (size_t)i * selt + s;
      const int j = nl_j[slot];
      if (j < 0) continue;
      const double* go = g.data() + 3 * slot;
      const double* r = rij + 3 * slot;
      for (int c = 0; c < 3; ++c) {
        f[3 * (size_t)i + c] += go[c];
        f[3 * (size_t)j + c] -= go[c];
      }
      for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b) {
          v[3 * a + b] -= go[a] * r[b];
          av[9 * (size_t)j + 3 * a + b] -= go[a] * r[b];
        }
    }
  }
  *energy = e;
  std::memcpy(force, f.data(), sizeof(double) * f.size());
  std::memcpy(virial, v, sizeof(v));
  if (atom_e) std::memcpy(atom_e, ae.data(), sizeof(double) * nloc);
  if (atom_virial) std::memcpy(atom_virial, av.data(), sizeof(double) * av.size());
  if (edge_grad) std::memcpy(edge_grad, g.data(), sizeof(double) * g.size());
  return 0;
}

}  // extern "C"
