// CPU oracle for the DPA4C-style (se_e2_a type) energy / force / virial path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
// compared against (tests/, __graft_entry__.smoke() and bench.py's timed CPU
// baseline).  Nothing in the product links or calls it.
//
// Parity status: UNPINNED.  The reference repository holds no implementation
// of this model family: its se_e2_a operators live in the un-vendored
// DeePMD-kit tarball pinned at 46fdc3e8b0c92524e85dad48ee00a8555a0a7595
// (production/dpa4c-runtime/third_party/sources.lock.json:4-12) and the only
// caller contract present is PL/pair_deepmd.cpp:370-371 -> deep_pot.compute().
// The math below restates the published DeepPot-SE definition (Zhang et al.,
// NeurIPS 2018) and DeePMD-kit's documented conventions; it is checked by
// finite differences, symmetry tests and an independent autograd restatement
// (tests/test_oracle.py), not against reference numbers (none exist).
//
// Conventions (fixed so the GPU path can be compared bit for bit):
//  * neighbour of local centre i: (j, n) with r_ijn = x'_j + n.B - x'_i and
//    |r| < rcut, where x' are coordinates wrapped into the cell (periodic
//    mode) or the raw coordinates with n = 0 (ghost mode, nghost > 0);
//  * per neighbour type t, candidates sorted by (r^2, j, image code) and the
//    first sel[t] kept, placed at offset sum(sel[:t]) of the row, -1 padding;
//  * r^2 = (dx*dx + dy*dy) + dz*dz with dx = (x'_j + s_x) - x'_i, all fp64,
//    no contraction (compile with -ffp-contract=off);
//  * edge gradient g = dE/dr_ij; F_i += g, F_j -= g; virial[a][b] and the
//    atom virial of j accumulate -g_a * r_b.  This is the sign and ownership
//    convention of the reference's edge assembly
//    (components/deepmd-op/overlays/op/pt/edge_force_virial.cu:8-11).
#include <omp.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

namespace {

struct Layer {
  int din = 0, dout = 0;
  std::vector<double> w, b;
};

struct Model {
  int ntypes = 0, axis = 0, type_one_side = 1, activation = 0;
  std::vector<int> emb, fit, sel;
  double rcut = 0, rcut_smth = 0;
  std::vector<double> bias;
  std::vector<std::vector<Layer>> emb_nets, fit_nets;
  int sel_total() const {
    int s = 0;
    for (int v : sel) s += v;
    return s;
  }
  int m1() const { return emb.back(); }
  int dim() const { return emb.back() * axis; }
};

std::string g_error;

bool read_model(const char* path, Model& m) {
  std::ifstream f(path, std::ios::binary);
  if (!f) {
    g_error = std::string("cannot open ") + path;
    return false;
  }
  std::vector<char> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  size_t off = 0;
  auto need = [&](size_t n) { return off + n <= buf.size(); };
  auto rd_i = [&]() {
    int32_t v = 0;
    if (need(4)) std::memcpy(&v, buf.data() + off, 4);
    off += 4;
    return (int)v;
  };
  auto rd_d = [&]() {
    double v = 0;
    if (need(8)) std::memcpy(&v, buf.data() + off, 8);
    off += 8;
    return v;
  };
  if (buf.size() < 8 || std::memcmp(buf.data(), "B2DPSEA1", 8) != 0) {
    g_error = "bad magic";
    return false;
  }
  off = 8;
  if (rd_i() != 1) {
    g_error = "bad version";
    return false;
  }
  m.ntypes = rd_i();
  int ne = rd_i();
  for (int i = 0; i < ne; ++i) m.emb.push_back(rd_i());
  m.axis = rd_i();
  int nf = rd_i();
  for (int i = 0; i < nf; ++i) m.fit.push_back(rd_i());
  m.type_one_side = rd_i();
  m.activation = rd_i();
  for (int i = 0; i < m.ntypes; ++i) m.sel.push_back(rd_i());
  m.rcut = rd_d();
  m.rcut_smth = rd_d();
  for (int i = 0; i < m.ntypes; ++i) m.bias.push_back(rd_d());
  auto rd_net = [&](const std::vector<int>& dims) {
    std::vector<Layer> net;
    for (size_t l = 0; l + 1 < dims.size(); ++l) {
      Layer L;
      L.din = dims[l];
      L.dout = dims[l + 1];
      L.w.resize((size_t)L.din * L.dout);
      L.b.resize(L.dout);
      for (auto& v : L.w) v = rd_d();
      for (auto& v : L.b) v = rd_d();
      net.push_back(std::move(L));
    }
    return net;
  };
  std::vector<int> ed{1};
  for (int v : m.emb) ed.push_back(v);
  int nnets = m.type_one_side ? m.ntypes : m.ntypes * m.ntypes;
  for (int i = 0; i < nnets; ++i) m.emb_nets.push_back(rd_net(ed));
  std::vector<int> fd{m.dim()};
  for (int v : m.fit) fd.push_back(v);
  fd.push_back(1);
  for (int i = 0; i < m.ntypes; ++i) m.fit_nets.push_back(rd_net(fd));
  if (off != buf.size()) {
    g_error = "model size mismatch";
    return false;
  }
  return true;
}

// ---------------------------------------------------------------- geometry
struct Cell {
  double B[3][3];     // rows are cell vectors
  double Binv[3][3];  // x = s.B  <=>  s = x.Binv
  double width[3];    // perpendicular widths
};

void make_cell(const double* box, Cell& c) {
  for (int a = 0; a < 3; ++a)
    for (int b = 0; b < 3; ++b) c.B[a][b] = box[3 * a + b];
  const double(*B)[3] = c.B;
  // Cofactor inverse, fixed operation order.
  double c00 = B[1][1] * B[2][2] - B[1][2] * B[2][1];
  double c01 = B[1][2] * B[2][0] - B[1][0] * B[2][2];
  double c02 = B[1][0] * B[2][1] - B[1][1] * B[2][0];
  double det = (B[0][0] * c00 + B[0][1] * c01) + B[0][2] * c02;
  double id = 1.0 / det;
  c.Binv[0][0] = c00 * id;
  c.Binv[1][0] = c01 * id;
  c.Binv[2][0] = c02 * id;
  c.Binv[0][1] = (B[0][2] * B[2][1] - B[0][1] * B[2][2]) * id;
  c.Binv[1][1] = (B[0][0] * B[2][2] - B[0][2] * B[2][0]) * id;
  c.Binv[2][1] = (B[0][1] * B[2][0] - B[0][0] * B[2][1]) * id;
  c.Binv[0][2] = (B[0][1] * B[1][2] - B[0][2] * B[1][1]) * id;
  c.Binv[1][2] = (B[0][2] * B[1][0] - B[0][0] * B[1][2]) * id;
  c.Binv[2][2] = (B[0][0] * B[1][1] - B[0][1] * B[1][0]) * id;
  double vol = std::fabs(det);
  for (int d = 0; d < 3; ++d) {
    const double* u = B[(d + 1) % 3];
    const double* v = B[(d + 2) % 3];
    double x = u[1] * v[2] - u[2] * v[1], y = u[2] * v[0] - u[0] * v[2], z = u[0] * v[1] - u[1] * v[0];
    c.width[d] = vol / std::sqrt(x * x + y * y + z * z);
  }
}

inline void frac(const Cell& c, const double* x, double* s) {
  for (int d = 0; d < 3; ++d) s[d] = (x[0] * c.Binv[0][d] + x[1] * c.Binv[1][d]) + x[2] * c.Binv[2][d];
}

inline int image_code(int n0, int n1, int n2) {
  return ((n0 + 512) << 20) | ((n1 + 512) << 10) | (n2 + 512);
}

struct Cand {
  double r2;
  int j, code;
  double r[3];
};

struct NL {
  int nloc = 0, selt = 0, ntypes = 0;
  std::vector<int> j, code, cnt;
  std::vector<double> rij;
  long overflow = 0;
};

// Builds the canonical neighbour list (see the conventions at the top).
bool build_nlist(int nloc, int nall, const double* coord, const int* atype, const double* box, double rcut,
                 int ntypes, const int* sel, NL& out) {
  const bool periodic = (box != nullptr) && (nall == nloc);
  int selt = 0;
  std::vector<int> off(ntypes + 1, 0);
  for (int t = 0; t < ntypes; ++t) {
    off[t + 1] = off[t] + sel[t];
  }
  selt = off[ntypes];
  out.nloc = nloc;
  out.selt = selt;
  out.ntypes = ntypes;
  out.j.assign((size_t)nloc * selt, -1);
  out.code.assign((size_t)nloc * selt, image_code(0, 0, 0));
  out.rij.assign((size_t)nloc * selt * 3, 0.0);
  out.cnt.assign((size_t)nloc * ntypes, 0);
  out.overflow = 0;
  const double rc2 = rcut * rcut;

  std::vector<double> xw((size_t)nall * 3);
  Cell cell{};
  int ncell[3] = {1, 1, 1}, reach[3] = {1, 1, 1};
  double lo[3] = {0, 0, 0}, hsz[3] = {1, 1, 1};
  std::vector<int> cell_of(nall);
  if (periodic) {
    make_cell(box, cell);
    for (int i = 0; i < nall; ++i) {
      double s[3];
      frac(cell, coord + 3 * i, s);
      double f[3] = {std::floor(s[0]), std::floor(s[1]), std::floor(s[2])};
      for (int c = 0; c < 3; ++c)
        xw[3 * i + c] = coord[3 * i + c] - ((f[0] * cell.B[0][c] + f[1] * cell.B[1][c]) + f[2] * cell.B[2][c]);
    }
    for (int d = 0; d < 3; ++d) {
      ncell[d] = std::max(1, (int)std::floor(cell.width[d] / rcut));
      reach[d] = (int)std::ceil(rcut * ncell[d] / cell.width[d] * (1.0 + 1e-12));
    }
    for (int i = 0; i < nall; ++i) {
      double s[3];
      frac(cell, &xw[3 * i], s);
      int ci[3];
      for (int d = 0; d < 3; ++d) ci[d] = std::min(ncell[d] - 1, std::max(0, (int)std::floor(s[d] * ncell[d])));
      cell_of[i] = (ci[0] * ncell[1] + ci[1]) * ncell[2] + ci[2];
    }
  } else {
    std::copy(coord, coord + (size_t)nall * 3, xw.begin());
    double hi[3];
    for (int d = 0; d < 3; ++d) {
      lo[d] = 1e300;
      hi[d] = -1e300;
    }
    for (int i = 0; i < nall; ++i)
      for (int d = 0; d < 3; ++d) {
        lo[d] = std::min(lo[d], coord[3 * i + d]);
        hi[d] = std::max(hi[d], coord[3 * i + d]);
      }
    for (int d = 0; d < 3; ++d) {
      double ext = std::max(hi[d] - lo[d], 1e-9);
      ncell[d] = std::max(1, (int)std::floor(ext / rcut));
      hsz[d] = ext / ncell[d];
      reach[d] = 1;
    }
    for (int i = 0; i < nall; ++i) {
      int ci[3];
      for (int d = 0; d < 3; ++d)
        ci[d] = std::min(ncell[d] - 1, std::max(0, (int)std::floor((coord[3 * i + d] - lo[d]) / hsz[d])));
      cell_of[i] = (ci[0] * ncell[1] + ci[1]) * ncell[2] + ci[2];
    }
  }
  const int ntot = ncell[0] * ncell[1] * ncell[2];
  std::vector<std::vector<int>> members(ntot);
  for (int i = 0; i < nall; ++i) members[cell_of[i]].push_back(i);

  long overflow = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : overflow)
  for (int i = 0; i < nloc; ++i) {
    int cc = cell_of[i];
    int ci[3] = {cc / (ncell[1] * ncell[2]), (cc / ncell[2]) % ncell[1], cc % ncell[2]};
    std::vector<std::vector<Cand>> per(ntypes);
    const double* xi = &xw[3 * i];
    for (int d0 = -reach[0]; d0 <= reach[0]; ++d0)
      for (int d1 = -reach[1]; d1 <= reach[1]; ++d1)
        for (int d2 = -reach[2]; d2 <= reach[2]; ++d2) {
          int u[3] = {ci[0] + d0, ci[1] + d1, ci[2] + d2};
          int img[3] = {0, 0, 0};
          bool skip = false;
          for (int d = 0; d < 3; ++d) {
            if (periodic) {
              int q = u[d] >= 0 ? u[d] / ncell[d] : -((-u[d] + ncell[d] - 1) / ncell[d]);
              img[d] = q;
              u[d] -= q * ncell[d];
            } else if (u[d] < 0 || u[d] >= ncell[d]) {
              skip = true;
            }
          }
          if (skip) continue;
          double sh[3] = {0, 0, 0};
          if (periodic)
            for (int c = 0; c < 3; ++c)
              sh[c] = ((double)img[0] * cell.B[0][c] + (double)img[1] * cell.B[1][c]) + (double)img[2] * cell.B[2][c];
          int code = image_code(img[0], img[1], img[2]);
          for (int j : members[(u[0] * ncell[1] + u[1]) * ncell[2] + u[2]]) {
            if (j == i && img[0] == 0 && img[1] == 0 && img[2] == 0) continue;
            const double* xj = &xw[3 * j];
            double r[3];
            for (int c = 0; c < 3; ++c) r[c] = (xj[c] + sh[c]) - xi[c];
            double r2 = (r[0] * r[0] + r[1] * r[1]) + r[2] * r[2];
            if (r2 < rc2) {
              int t = atype[j];
              if (t < 0 || t >= ntypes) continue;
              per[t].push_back(Cand{r2, j, code, {r[0], r[1], r[2]}});
            }
          }
        }
    for (int t = 0; t < ntypes; ++t) {
      auto& v = per[t];
      std::sort(v.begin(), v.end(), [](const Cand& a, const Cand& b) {
        if (a.r2 != b.r2) return a.r2 < b.r2;
        if (a.j != b.j) return a.j < b.j;
        return a.code < b.code;
      });
      int keep = std::min<int>((int)v.size(), sel[t]);
      if ((int)v.size() > sel[t]) overflow += (long)v.size() - sel[t];
      out.cnt[(size_t)i * ntypes + t] = keep;
      for (int s = 0; s < keep; ++s) {
        size_t slot = (size_t)i * selt + off[t] + s;
        out.j[slot] = v[s].j;
        out.code[slot] = v[s].code;
        for (int c = 0; c < 3; ++c) out.rij[3 * slot + c] = v[s].r[c];
      }
    }
  }
  out.overflow = overflow;
  return true;
}

// ---------------------------------------------------------------- model math
// Smooth switch of DeePMD's env_mat_a: 1 below rs, quintic to 0 at rc.
inline void switch_fn(double r, double rs, double rc, double& sw, double& dsw) {
  if (r < rs) {
    sw = 1.0;
    dsw = 0.0;
  } else if (r < rc) {
    double du = 1.0 / (rc - rs);
    double u = (r - rs) * du;
    double u2 = u * u, u3 = u2 * u;
    sw = u3 * (-6.0 * u2 + 15.0 * u - 10.0) + 1.0;
    dsw = (3.0 * u2 * (-6.0 * u2 + 15.0 * u - 10.0) + u3 * (-12.0 * u + 15.0)) * du;
  } else {
    sw = 0.0;
    dsw = 0.0;
  }
}

// Embedding net forward for scalar input; stores every layer output.
// Residual rule of DeePMD's embedding_net: d_out == d_in -> x + h;
// d_out == 2 d_in -> concat(x, x) + h; otherwise h.
void emb_forward(const std::vector<Layer>& net, double s, std::vector<std::vector<double>>& act) {
  act.resize(net.size() + 1);
  act[0].assign(1, s);
  for (size_t l = 0; l < net.size(); ++l) {
    const Layer& L = net[l];
    const auto& x = act[l];
    auto& y = act[l + 1];
    y.assign(L.dout, 0.0);
    for (int n = 0; n < L.dout; ++n) {
      double z = L.b[n];
      for (int k = 0; k < L.din; ++k) z += x[k] * L.w[(size_t)k * L.dout + n];
      double h = std::tanh(z);
      if (L.dout == L.din)
        h += x[n];
      else if (L.dout == 2 * L.din)
        h += x[n % L.din];
      y[n] = h;
    }
  }
}

// Backward through the embedding net: dy (last layer) -> d(input).
double emb_backward(const std::vector<Layer>& net, const std::vector<std::vector<double>>& act,
                    std::vector<double> dy) {
  for (int l = (int)net.size() - 1; l >= 0; --l) {
    const Layer& L = net[l];
    const auto& x = act[l];
    const auto& y = act[l + 1];
    std::vector<double> dx(L.din, 0.0);
    for (int n = 0; n < L.dout; ++n) {
      // tanh part: h = y - residual
      double res = 0.0;
      if (L.dout == L.din)
        res = x[n];
      else if (L.dout == 2 * L.din)
        res = x[n % L.din];
      double h = y[n] - res;
      double dz = dy[n] * (1.0 - h * h);
      for (int k = 0; k < L.din; ++k) dx[k] += dz * L.w[(size_t)k * L.dout + n];
      if (L.dout == L.din)
        dx[n] += dy[n];
      else if (L.dout == 2 * L.din)
        dx[n % L.din] += dy[n];
    }
    dy.swap(dx);
  }
  return dy[0];
}

// Fitting net forward + input gradient.  Residual when width is unchanged
// (DeePMD fitting rule); last layer is linear.
double fit_forward_backward(const std::vector<Layer>& net, const std::vector<double>& d, std::vector<double>& dd) {
  std::vector<std::vector<double>> act(net.size() + 1);
  std::vector<std::vector<double>> th(net.size());
  act[0] = d;
  for (size_t l = 0; l < net.size(); ++l) {
    const Layer& L = net[l];
    const auto& x = act[l];
    auto& y = act[l + 1];
    y.assign(L.dout, 0.0);
    th[l].assign(L.dout, 0.0);
    bool last = (l + 1 == net.size());
    for (int n = 0; n < L.dout; ++n) {
      double z = L.b[n];
      for (int k = 0; k < L.din; ++k) z += x[k] * L.w[(size_t)k * L.dout + n];
      if (last) {
        y[n] = z;
      } else {
        double h = std::tanh(z);
        th[l][n] = h;
        y[n] = (l >= 1 && L.dout == L.din) ? x[n] + h : h;
      }
    }
  }
  double e = act.back()[0];
  std::vector<double> dy(1, 1.0);
  for (int l = (int)net.size() - 1; l >= 0; --l) {
    const Layer& L = net[l];
    bool last = (l + 1 == (int)net.size());
    bool res = (!last && l >= 1 && L.dout == L.din);
    std::vector<double> dx(L.din, 0.0);
    for (int n = 0; n < L.dout; ++n) {
      double dz = last ? dy[n] : dy[n] * (1.0 - th[l][n] * th[l][n]);
      for (int k = 0; k < L.din; ++k) dx[k] += dz * L.w[(size_t)k * L.dout + n];
      if (res) dx[n] += dy[n];
    }
    dy.swap(dx);
  }
  dd = dy;
  return e;
}

struct Handle {
  Model m;
};

}  // namespace

extern "C" {

const char* oracle_last_error() { return g_error.c_str(); }

void* oracle_load(const char* path) {
  auto* h = new Handle;
  if (!read_model(path, h->m)) {
    delete h;
    return nullptr;
  }
  return h;
}

void oracle_free(void* h) { delete static_cast<Handle*>(h); }

int oracle_set_threads(int n) {
  if (n > 0) omp_set_num_threads(n);
  return omp_get_max_threads();
}

// Canonical neighbour list.  nlist/code: [nloc*selt]; rij: [nloc*selt*3];
// counts: [nloc*ntypes].  Returns the number of candidates dropped by sel.
long oracle_nlist(int nloc, int nall, const double* coord, const int* atype, const double* box, double rcut,
                  int ntypes, const int* sel, int* nlist, int* code, double* rij, int* counts) {
  NL nl;
  build_nlist(nloc, nall, coord, atype, box, rcut, ntypes, sel, nl);
  std::copy(nl.j.begin(), nl.j.end(), nlist);
  if (code) std::copy(nl.code.begin(), nl.code.end(), code);
  if (rij) std::copy(nl.rij.begin(), nl.rij.end(), rij);
  if (counts) std::copy(nl.cnt.begin(), nl.cnt.end(), counts);
  return nl.overflow;
}

// Energy, forces and virial.  force / atom_virial have nall rows (periodic
// mode: nall == nloc and image contributions fold onto the owning atom).
// descriptor (optional): [nloc, M1*axis]; grad_descriptor (optional) the same.
int oracle_compute(void* hp, int nloc, int nall, const double* coord, const int* atype, const double* box,
                   double* energy, double* force, double* virial, double* atom_energy, double* atom_virial,
                   double* descriptor, double* grad_descriptor, long* overflow_out) {
  const Model& m = static_cast<Handle*>(hp)->m;
  NL nl;
  build_nlist(nloc, nall, coord, atype, box, m.rcut, m.ntypes, m.sel.data(), nl);
  if (overflow_out) *overflow_out = nl.overflow;
  const int selt = nl.selt, M1 = m.m1(), M2 = m.axis, ntypes = m.ntypes;
  const double inv_nnei = 1.0 / (double)selt;
  std::vector<int> off(ntypes + 1, 0);
  for (int t = 0; t < ntypes; ++t) off[t + 1] = off[t] + m.sel[t];
  std::vector<double> gedge((size_t)nloc * selt * 3, 0.0);
  std::vector<double> eatom(nloc, 0.0);

#pragma omp parallel for schedule(dynamic, 16)
  for (int i = 0; i < nloc; ++i) {
    const int ti = atype[i];
    std::vector<double> T((size_t)4 * M1, 0.0);
    // forward: env + embedding + contraction
    struct Edge {
      double rt[4], drt[4][3];
      std::vector<std::vector<double>> act;
      int net;
      size_t slot;
    };
    std::vector<Edge> edges;
    for (int t = 0; t < ntypes; ++t) {
      int cnt = nl.cnt[(size_t)i * ntypes + t];
      int net = m.type_one_side ? t : ti * ntypes + t;
      for (int s = 0; s < cnt; ++s) {
        size_t slot = (size_t)i * selt + off[t] + s;
        const double* r = &nl.rij[3 * slot];
        double r2 = (r[0] * r[0] + r[1] * r[1]) + r[2] * r[2];
        double rr = std::sqrt(r2);
        double sw, dsw;
        switch_fn(rr, m.rcut_smth, m.rcut, sw, dsw);
        Edge e;
        e.net = net;
        e.slot = slot;
        double inv_r = 1.0 / rr, inv_r2 = inv_r * inv_r;
        e.rt[0] = sw * inv_r;
        for (int c = 0; c < 3; ++c) e.rt[1 + c] = sw * r[c] * inv_r2;
        // d rt / d r_c
        double d0 = (dsw * inv_r - sw * inv_r2);  // d(sw/r)/dr
        for (int c = 0; c < 3; ++c) e.drt[0][c] = d0 * r[c] * inv_r;
        for (int a = 0; a < 3; ++a)
          for (int c = 0; c < 3; ++c) {
            // d(sw r_a / r^2)/d r_c
            double v = dsw * r[c] * inv_r * r[a] * inv_r2 + sw * ((a == c ? inv_r2 : 0.0) - 2.0 * r[a] * r[c] * inv_r2 * inv_r2);
            e.drt[1 + a][c] = v;
          }
        emb_forward(m.emb_nets[net], e.rt[0], e.act);
        const auto& G = e.act.back();
        for (int k = 0; k < 4; ++k)
          for (int a = 0; a < M1; ++a) T[(size_t)k * M1 + a] += e.rt[k] * G[a];
        edges.push_back(std::move(e));
      }
    }
    for (auto& v : T) v *= inv_nnei;
    std::vector<double> D((size_t)M1 * M2);
    for (int a = 0; a < M1; ++a)
      for (int b = 0; b < M2; ++b) {
        double acc = 0.0;
        for (int k = 0; k < 4; ++k) acc += T[(size_t)k * M1 + a] * T[(size_t)k * M1 + b];
        D[(size_t)a * M2 + b] = acc;
      }
    std::vector<double> dD;
    double ei = fit_forward_backward(m.fit_nets[ti], D, dD) + m.bias[ti];
    eatom[i] = ei;
    if (descriptor) std::copy(D.begin(), D.end(), descriptor + (size_t)i * M1 * M2);
    if (grad_descriptor) std::copy(dD.begin(), dD.end(), grad_descriptor + (size_t)i * M1 * M2);
    // dT[k][a] = sum_b dD[a][b] T[k][b] + [a < M2] sum_c dD[c][a] T[k][c]
    std::vector<double> dT((size_t)4 * M1, 0.0);
    for (int k = 0; k < 4; ++k)
      for (int a = 0; a < M1; ++a) {
        double acc = 0.0;
        for (int b = 0; b < M2; ++b) acc += dD[(size_t)a * M2 + b] * T[(size_t)k * M1 + b];
        if (a < M2)
          for (int c = 0; c < M1; ++c) acc += dD[(size_t)c * M2 + a] * T[(size_t)k * M1 + c];
        dT[(size_t)k * M1 + a] = acc;
      }
    for (auto& e : edges) {
      const auto& G = e.act.back();
      std::vector<double> dG(M1, 0.0);
      double drt[4] = {0, 0, 0, 0};
      for (int a = 0; a < M1; ++a) {
        double acc = 0.0;
        for (int k = 0; k < 4; ++k) {
          acc += dT[(size_t)k * M1 + a] * e.rt[k];
          drt[k] += dT[(size_t)k * M1 + a] * G[a];
        }
        dG[a] = acc * inv_nnei;
      }
      for (int k = 0; k < 4; ++k) drt[k] *= inv_nnei;
      drt[0] += emb_backward(m.emb_nets[e.net], e.act, dG);
      for (int c = 0; c < 3; ++c) {
        double g = 0.0;
        for (int k = 0; k < 4; ++k) g += drt[k] * e.drt[k][c];
        gedge[3 * e.slot + c] = g;
      }
    }
  }

  // Assembly (serial, fixed order).
  double etot = 0.0;
  for (int i = 0; i < nloc; ++i) etot += eatom[i];
  if (energy) *energy = etot;
  if (atom_energy) std::copy(eatom.begin(), eatom.end(), atom_energy);
  std::vector<double> F((size_t)nall * 3, 0.0), AV((size_t)nall * 9, 0.0);
  double W[9] = {0};
  for (int i = 0; i < nloc; ++i)
    for (int s = 0; s < selt; ++s) {
      size_t slot = (size_t)i * selt + s;
      int j = nl.j[slot];
      if (j < 0) continue;
      const double* g = &gedge[3 * slot];
      const double* r = &nl.rij[3 * slot];
      for (int c = 0; c < 3; ++c) {
        F[3 * (size_t)i + c] += g[c];
        F[3 * (size_t)j + c] -= g[c];
      }
      for (int a = 0; a < 3; ++a)
        for (int b = 0; b < 3; ++b) {
          double v = -g[a] * r[b];
          W[3 * a + b] += v;
          AV[9 * (size_t)j + 3 * a + b] += v;
        }
    }
  if (force) std::copy(F.begin(), F.end(), force);
  if (virial) std::copy(W, W + 9, virial);
  if (atom_virial) std::copy(AV.begin(), AV.end(), atom_virial);
  return 0;
}

}  // extern "C"
