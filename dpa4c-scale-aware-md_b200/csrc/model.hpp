// Host-side model description and loader for the B2DPSEA1 model file.
//
// The file layout is written by modelgen.py (same directory as the package):
// magic "B2DPSEA1", int32 header (version, ntypes, embedding widths, axis,
// fitting widths, type_one_side, activation, sel), fp64 rcut, rcut_smth,
// bias_atom_e, then the embedding nets and fitting nets, each layer as
// W[d_in][d_out] row-major followed by b[d_out].
#pragma once

#include <cstdint>
#include <cstring>
#include <fstream>
#include <iterator>
#include <string>
#include <vector>

namespace b200dp {

struct HostLayer {
  int din = 0, dout = 0;
  std::vector<double> w, b;
};

struct HostModel {
  int ntypes = 0, axis = 0, type_one_side = 1, activation = 0;
  std::vector<int> emb, fit, sel;
  double rcut = 0, rcut_smth = 0;
  std::vector<double> bias_atom_e;
  std::vector<std::vector<HostLayer>> emb_nets;  // [n_emb_nets][layers]
  std::vector<std::vector<HostLayer>> fit_nets;  // [ntypes][layers incl. final linear]

  int sel_total() const {
    int s = 0;
    for (int v : sel) s += v;
    return s;
  }
  int m1() const { return emb.empty() ? 0 : emb.back(); }
  int dim() const { return m1() * axis; }
  int n_emb_nets() const { return type_one_side ? ntypes : ntypes * ntypes; }
};

// Returns an empty string on success, else a message.
inline std::string load_model(const char* path, HostModel& m) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return std::string("cannot open model file ") + path;
  std::vector<char> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  size_t off = 0;
  bool short_read = false;
  auto rd = [&](void* dst, size_t n) {
    if (off + n > buf.size()) {
      short_read = true;
      std::memset(dst, 0, n);
    } else {
      std::memcpy(dst, buf.data() + off, n);
    }
    off += n;
  };
  auto rd_i = [&]() {
    int32_t v;
    rd(&v, 4);
    return (int)v;
  };
  auto rd_d = [&]() {
    double v;
    rd(&v, 8);
    return v;
  };
  if (buf.size() < 8 || std::memcmp(buf.data(), "B2DPSEA1", 8) != 0) return "model file: bad magic";
  off = 8;
  if (rd_i() != 1) return "model file: unsupported version";
  m.ntypes = rd_i();
  int ne = rd_i();
  if (m.ntypes <= 0 || m.ntypes > 8 || ne <= 0 || ne > 6) return "model file: bad header";
  for (int i = 0; i < ne; ++i) m.emb.push_back(rd_i());
  m.axis = rd_i();
  int nf = rd_i();
  if (nf <= 0 || nf > 5) return "model file: bad fitting depth";
  for (int i = 0; i < nf; ++i) m.fit.push_back(rd_i());
  m.type_one_side = rd_i();
  m.activation = rd_i();
  for (int i = 0; i < m.ntypes; ++i) m.sel.push_back(rd_i());
  m.rcut = rd_d();
  m.rcut_smth = rd_d();
  for (int i = 0; i < m.ntypes; ++i) m.bias_atom_e.push_back(rd_d());
  if (short_read) return "model file: truncated header";
  for (int v : m.emb)
    if (v <= 0 || v > 256) return "model file: embedding width out of range (1..256)";
  for (int v : m.fit)
    if (v <= 0 || v > 4096) return "model file: fitting width out of range";
  if (m.axis <= 0 || m.axis > m.m1()) return "model file: axis must be in [1, embedding width]";
  if (m.activation != 0) return "model file: only tanh activation is supported";
  if (!(m.rcut > m.rcut_smth && m.rcut_smth >= 0)) return "model file: need rcut > rcut_smth >= 0";
  auto rd_net = [&](const std::vector<int>& dims) {
    std::vector<HostLayer> net;
    for (size_t l = 0; l + 1 < dims.size(); ++l) {
      HostLayer L;
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
  for (int i = 0; i < m.n_emb_nets(); ++i) m.emb_nets.push_back(rd_net(ed));
  std::vector<int> fd{m.dim()};
  for (int v : m.fit) fd.push_back(v);
  fd.push_back(1);
  for (int i = 0; i < m.ntypes; ++i) m.fit_nets.push_back(rd_net(fd));
  if (short_read) return "model file: truncated weights";
  if (off != buf.size()) return "model file: trailing bytes";
  return "";
}

// C8L2 model file (magic "B2DPC8L2"; layout written by modelgen.py's
// save_c8): int32 version, ntypes, channels, lmax, interval_count,
// table_width, n_fit, fit[n_fit], resnets[n_fit], activation, sel[ntypes];
// fp64 table_stride, table_max, rcut, eps, degree_floor, b_head,
// bias_atom_e[ntypes]; fp64 table [interval_count][6 * table_width],
// pair_film [ntypes^2][channels][2], type_embedding [ntypes][channels],
// readout [8][4][4], output_mean [70], output_inv_std [70]; fitting layers
// (W [d_in][d_out], b [d_out]) from the 70-wide descriptor; w_head.
struct C8Host {
  int ntypes = 0, channels = 0, lmax = 0, nint = 0, width = 0, act = 1;
  std::vector<int> fit, res, sel;
  double stride = 0, tmax = 0, rcut = 0, eps = 0, floor_ = 0, b_head = 0;
  std::vector<double> bias, table, film, temb, readout, mean, istd, w_head;
  std::vector<HostLayer> layers;
};

inline bool is_c8_model(const char* path) {
  std::ifstream f(path, std::ios::binary);
  char magic[8] = {};
  return f && f.read(magic, 8) && std::memcmp(magic, "B2DPC8L2", 8) == 0;
}

inline std::string load_c8_model(const char* path, C8Host& m) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return std::string("cannot open model file ") + path;
  std::vector<char> buf((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  size_t off = 0;
  bool short_read = false;
  auto rd = [&](void* dst, size_t n) {
    if (off + n > buf.size()) {
      short_read = true;
      std::memset(dst, 0, n);
    } else {
      std::memcpy(dst, buf.data() + off, n);
    }
    off += n;
  };
  auto rd_i = [&]() {
    int32_t v;
    rd(&v, 4);
    return (int)v;
  };
  auto rd_v = [&](std::vector<double>& v, size_t n) {
    v.resize(n);
    if (n) rd(v.data(), 8 * n);
  };
  if (buf.size() < 8 || std::memcmp(buf.data(), "B2DPC8L2", 8) != 0) return "model file: bad magic";
  off = 8;
  if (rd_i() != 1) return "model file: unsupported version";
  m.ntypes = rd_i();
  m.channels = rd_i();
  m.lmax = rd_i();
  m.nint = rd_i();
  m.width = rd_i();
  const int nf = rd_i();
  if (m.ntypes <= 0 || m.ntypes > 8) return "model file: ntypes out of range (1..8)";
  if (m.channels != 8 || m.lmax != 2 || m.width != 8)
    return "model file: only the C8 L2 profile (8 channels, lmax 2, table width 8) is supported";
  if (nf <= 0 || nf > 4 || m.nint <= 0) return "model file: bad C8L2 header";
  for (int i = 0; i < nf; ++i) m.fit.push_back(rd_i());
  for (int i = 0; i < nf; ++i) m.res.push_back(rd_i());
  m.act = rd_i();
  for (int t = 0; t < m.ntypes; ++t) m.sel.push_back(rd_i());
  double d[6];
  rd(d, sizeof(d));
  m.stride = d[0], m.tmax = d[1], m.rcut = d[2], m.eps = d[3], m.floor_ = d[4], m.b_head = d[5];
  rd_v(m.bias, m.ntypes);
  if (short_read) return "model file: truncated header";
  for (int v : m.fit)
    if (v <= 0 || v > 256) return "model file: fitting width out of range (1..256)";
  if (m.act != 0 && m.act != 1) return "model file: activation must be 0 (tanh) or 1 (SiLU)";
  if (!(m.rcut > 0) || !(m.stride > 0) || !(m.floor_ >= 0)) return "model file: bad radial parameters";
  rd_v(m.table, (size_t)m.nint * 6 * m.width);
  rd_v(m.film, (size_t)m.ntypes * m.ntypes * m.channels * 2);
  rd_v(m.temb, (size_t)m.ntypes * m.channels);
  rd_v(m.readout, 8 * 16);
  rd_v(m.mean, 70);
  rd_v(m.istd, 70);
  int din = 70;
  for (int l = 0; l < nf; ++l) {
    HostLayer L;
    L.din = din;
    L.dout = m.fit[l];
    rd_v(L.w, (size_t)L.din * L.dout);
    rd_v(L.b, L.dout);
    m.layers.push_back(std::move(L));
    din = m.fit[l];
  }
  rd_v(m.w_head, din);
  if (short_read) return "model file: truncated weights";
  if (off != buf.size()) return "model file: trailing bytes";
  return "";
}

}  // namespace b200dp
