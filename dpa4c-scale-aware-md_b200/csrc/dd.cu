// Domain-decomposed force evaluation and molecular dynamics over the GPUs of
// one node, one process per GPU, orchestrated in C++ (no Python, no torch).
//
// Replaces, for this hot path, what LAMMPS' Kokkos build does around the pair
// style in the reference: the atom exchange at reneighbouring
// (components/lammps/overlays/src/KOKKOS/comm_kokkos.cpp:809-1000,
// CommKokkos::exchange / exchange_device), the ghost-atom borders and the
// per-step forward / reverse communication
// (components/lammps-deepmd-plugin/src/pair_deepmd_kokkos.cpp:84-124, 931-993),
// and the fix nvt time integration with the chain on the device
// (components/lammps/overlays/src/KOKKOS/dpa_fast_step_kokkos.h:307-400).
//
// Layout: each rank owns the atoms of its sub-box (px x py x pz grid of the
// orthorhombic periodic box) and keeps a ghost shell of width `halo` built by
// the staged exchange along x, then y, then z (ghosts received in one
// dimension are forwarded in the next, which covers edges and corners).
//   * setup, atom migration and the ghost plan (host, at creation and every
//     `rebuild_every` MD steps): NCCL point-to-point messages, counts first;
//   * every step (device, no host synchronisation, capturable): the owners'
//     positions published into their exported buffers, a device-side
//     rendezvous, one kernel gathering the ghost rows over NVLink, the force
//     call whose assembly adds each ghost row's reverse contribution into the
//     owner's fixed-point accumulator, a rendezvous summing energy and virial
//     in rank order, and the owners' conversion of their accumulators.
// Everything a rank computes is deterministic: migrated atoms are kept in
// global-id order, the plan follows from positions, the fixed-point sums do
// not depend on arrival order and the rendezvous sums in rank order.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/b200dp.h"
#include "common.cuh"

namespace b200dp {
namespace {

#include "md_kernels.cuh"

// ---------------------------------------------------------------- transport
// Point-to-point messages between the ranks (host buffers).  Every rank posts
// the same sequence of calls, so messages between a pair match in order.
class Comm {
 public:
  virtual ~Comm() = default;
  // sends sb bytes to rank `to` and receives rb bytes from rank `from`
  virtual bool sendrecv(int to, const void* s, size_t sb, int from, void* r, size_t rb) = 0;
  int rank = 0, size = 1;
  bool allgather(const void* s, size_t b, void* r) {
    for (int q = 0; q < size; ++q) {  // round q: to rank + q, from rank - q
      const int to = (rank + q) % size, from = (rank - q + size) % size;
      if (!sendrecv(to, s, b, from, static_cast<char*>(r) + (size_t)from * b, b)) return false;
    }
    return true;
  }
  template <class T>
  bool exchange(int to, const std::vector<T>& out, int from, std::vector<T>& in) {
    long long ns = (long long)out.size(), nr = 0;
    if (!sendrecv(to, &ns, sizeof(ns), from, &nr, sizeof(nr)) || nr < 0) return false;
    in.resize((size_t)nr);
    return sendrecv(to, out.data(), sizeof(T) * out.size(), from, in.data(), sizeof(T) * in.size());
  }
};

// NCCL between the processes of a node; host data staged through one device buffer.
class NcclComm : public Comm {
 public:
  ncclComm_t comm = nullptr;
  cudaStream_t st = nullptr;
  char* dbuf = nullptr;
  size_t dcap = 0;
  ~NcclComm() override {
    if (dbuf) cudaFree(dbuf);
    if (comm) ncclCommDestroy(comm);
  }
  bool sendrecv(int to, const void* s, size_t sb, int from, void* r, size_t rb) override {
    if (to == rank && from == rank) {
      if (sb != rb) return false;
      if (sb) std::memcpy(r, s, sb);
      return true;
    }
    const size_t so = (sb + 255) & ~(size_t)255;
    if (so + rb > dcap) {
      if (dbuf) cudaFree(dbuf);
      dbuf = nullptr;
      dcap = std::max<size_t>(so + rb, 1 << 20);
      if (cudaMalloc(&dbuf, dcap) != cudaSuccess) {
        dcap = 0;
        return false;
      }
    }
    if (sb && cudaMemcpyAsync(dbuf, s, sb, cudaMemcpyHostToDevice, st) != cudaSuccess) return false;
    if (ncclGroupStart() != ncclSuccess) return false;
    ncclResult_t rs = ncclSuccess, rr = ncclSuccess;
    if (sb) rs = ncclSend(dbuf, sb, ncclChar, to, comm, st);
    if (rb) rr = ncclRecv(dbuf + so, rb, ncclChar, from, comm, st);
    // the group is closed whatever the two calls returned
    if (ncclGroupEnd() != ncclSuccess || rs != ncclSuccess || rr != ncclSuccess) return false;
    if (rb && cudaMemcpyAsync(r, dbuf + so, rb, cudaMemcpyDeviceToHost, st) != cudaSuccess) return false;
    return cudaStreamSynchronize(st) == cudaSuccess;
  }
};

// Threads of one process standing in for ranks (the CPU check of the plan).
struct Mailboxes {
  std::mutex m;
  std::condition_variable cv;
  int n = 0;
  std::vector<std::deque<std::vector<char>>> q;  // [from * n + to]
};
class ThreadComm : public Comm {
 public:
  Mailboxes* mb = nullptr;
  bool sendrecv(int to, const void* s, size_t sb, int from, void* r, size_t rb) override {
    if (to == rank && from == rank) {
      if (sb != rb) return false;
      if (sb) std::memcpy(r, s, sb);
      return true;
    }
    {
      std::lock_guard<std::mutex> lk(mb->m);
      const char* c = static_cast<const char*>(s);
      mb->q[(size_t)rank * mb->n + to].emplace_back(c, c + sb);
    }
    mb->cv.notify_all();
    std::unique_lock<std::mutex> lk(mb->m);
    auto& box = mb->q[(size_t)from * mb->n + rank];
    if (!mb->cv.wait_for(lk, std::chrono::seconds(60), [&] { return !box.empty(); })) return false;
    std::vector<char> msg = std::move(box.front());
    box.pop_front();
    if (msg.size() != rb) return false;
    if (rb) std::memcpy(r, msg.data(), rb);
    return true;
  }
};

// ---------------------------------------------------------------- decomposition
struct Decomp {
  int grid[3] = {1, 1, 1}, rank = 0, cell[3] = {0, 0, 0};
  double L[3] = {0, 0, 0}, lo[3] = {0, 0, 0}, hi[3] = {0, 0, 0}, halo = 0;
  const char* init(const double* box, const int* g, int r, double h) {
    for (int a = 0; a < 3; ++a)
      for (int b = 0; b < 3; ++b)
        if (a != b && box[3 * a + b] != 0.0) return "domain decomposition needs an orthorhombic box";
    for (int d = 0; d < 3; ++d) {
      grid[d] = g[d];
      L[d] = box[4 * d];
      if (grid[d] < 1 || !(L[d] > 0)) return "bad grid or box";
    }
    rank = r;
    cell[0] = r / (grid[1] * grid[2]);
    cell[1] = (r / grid[2]) % grid[1];
    cell[2] = r % grid[2];
    halo = h;
    for (int d = 0; d < 3; ++d) {
      const double w = L[d] / grid[d];
      lo[d] = cell[d] * w;
      hi[d] = (cell[d] + 1) * w;
      if (!(h > 0) || h > w) return "the halo must be positive and no wider than a sub-box";
    }
    return nullptr;
  }
  int rank_of(int c0, int c1, int c2) const {
    const int c[3] = {((c0 % grid[0]) + grid[0]) % grid[0], ((c1 % grid[1]) + grid[1]) % grid[1],
                      ((c2 % grid[2]) + grid[2]) % grid[2]};
    return (c[0] * grid[1] + c[1]) * grid[2] + c[2];
  }
  int neighbour(int dim, int dir) const {
    int c[3] = {cell[0], cell[1], cell[2]};
    c[dim] += dir;
    return rank_of(c[0], c[1], c[2]);
  }
  // shift for atoms sent in `dir` along `dim` (across the box edge)
  double send_shift(int dim, int dir) const {
    if (dir > 0 && cell[dim] == grid[dim] - 1) return -L[dim];
    if (dir < 0 && cell[dim] == 0) return L[dim];
    return 0.0;
  }
  // the box scaled by `r` about the origin (a barostat step): every bound scales with it
  void scale(double r) {
    for (int d = 0; d < 3; ++d) {
      L[d] *= r;
      lo[d] *= r;
      hi[d] *= r;
    }
  }
  bool owns(const double* w) const {
    for (int d = 0; d < 3; ++d)
      if (!(w[d] >= lo[d] && w[d] < hi[d])) return false;
    return true;
  }
};

// position wrapped into [0, L) (a rounding result of exactly L goes to 0)
double wrap1(double x, double L) {
  double w = x - std::floor(x / L) * L;
  if (w >= L) w -= L;
  return w;
}

struct Atom {  // an owned atom (host; 64 bytes)
  double x[3], v[3];
  long long id;
  int type, pad;
};
struct Ghost {  // a ghost row (host; 72 bytes)
  double x[3], shift[3];
  long long id;
  int type, org_rank, org_row, pad;
};

// Atoms that left the sub-box go to the face neighbour, dimension by
// dimension (an atom crossing an edge or corner travels in two or three
// hops); then every position is wrapped into the box and the atoms are kept
// in global-id order.  An atom may move at most one sub-box between calls.
const char* migrate(Comm& c, const Decomp& d, std::vector<Atom>& a) {
  for (int dim = 0; dim < 3; ++dim) {
    if (d.grid[dim] == 1) continue;
    std::vector<Atom> keep, down, up;
    keep.reserve(a.size());
    for (const Atom& at : a) {
      if (at.x[dim] < d.lo[dim])
        down.push_back(at);
      else if (at.x[dim] >= d.hi[dim])
        up.push_back(at);
      else
        keep.push_back(at);
    }
    for (int k = 0; k < 2; ++k) {
      const int dir = k == 0 ? -1 : 1;
      std::vector<Atom> in;
      if (!c.exchange(d.neighbour(dim, dir), k == 0 ? down : up, d.neighbour(dim, -dir), in))
        return "atom migration: exchange between ranks failed";
      keep.insert(keep.end(), in.begin(), in.end());
    }
    a.swap(keep);
  }
  for (Atom& at : a) {
    for (int dim = 0; dim < 3; ++dim) at.x[dim] = wrap1(at.x[dim], d.L[dim]);
    if (!d.owns(at.x)) return "an atom moved more than one sub-box between rebuilds";
  }
  std::sort(a.begin(), a.end(), [](const Atom& p, const Atom& q) { return p.id < q.id; });
  return nullptr;
}

// Ghost shell of the owned atoms by the staged exchange (both directions of
// a dimension select from the rows present before that dimension).  Every
// ghost records its owner (rank, row) and the periodic shift from the
// owner's position, each component the one pass shift applied to it.
const char* build_halo(Comm& c, const Decomp& d, const std::vector<Atom>& own, std::vector<Ghost>& out) {
  std::vector<Ghost> rows(own.size());
  for (size_t i = 0; i < own.size(); ++i) {
    Ghost& g = rows[i];
    std::memset(&g, 0, sizeof(g));
    for (int k = 0; k < 3; ++k) g.x[k] = own[i].x[k];
    g.id = own[i].id;
    g.type = own[i].type;
    g.org_rank = d.rank;
    g.org_row = (int)i;
  }
  for (int dim = 0; dim < 3; ++dim) {
    const size_t base = rows.size();
    std::vector<Ghost> blocks[2];
    for (int k = 0; k < 2; ++k) {
      const int dir = k == 0 ? -1 : 1;
      const double s = d.send_shift(dim, dir);
      std::vector<Ghost> send;
      for (size_t i = 0; i < base; ++i) {
        const double xd = rows[i].x[dim];
        const bool sel = dir > 0 ? xd >= d.hi[dim] - d.halo : xd < d.lo[dim] + d.halo;
        if (!sel) continue;
        Ghost g = rows[i];
        g.x[dim] += s;
        g.shift[dim] += s;
        send.push_back(g);
      }
      if (!c.exchange(d.neighbour(dim, dir), send, d.neighbour(dim, -dir), blocks[k]))
        return "ghost plan: exchange between ranks failed";
    }
    rows.insert(rows.end(), blocks[0].begin(), blocks[0].end());
    rows.insert(rows.end(), blocks[1].begin(), blocks[1].end());
  }
  out.assign(rows.begin() + (long)own.size(), rows.end());
  return nullptr;
}

template <class T>
struct DevArr {
  T* p = nullptr;
  size_t cap = 0;
  ~DevArr() {
    if (p) cudaFree(p);
  }
  cudaError_t ensure(size_t n) {
    if (n <= cap && p) return cudaSuccess;
    if (p) cudaFree(p);
    p = nullptr;
    cap = std::max<size_t>(n, 1);
    return cudaMalloc(&p, sizeof(T) * cap);
  }
};

// one warp: out[0] = sum of the partials in a fixed order
__global__ void k_dd_sum(const double* __restrict__ part, int n, double* __restrict__ out) {
  const double s = sum_parts(part, n);
  if (threadIdx.x == 0) out[0] = s;
}

}  // namespace
}  // namespace b200dp

using namespace b200dp;

struct b200dp_dd {
  b200dp_engine* engine = nullptr;
  int device = 0;
  std::unique_ptr<NcclComm> comm;
  Decomp dcmp;
  double region[6] = {0, 0, 0, 0, 0, 0};
  double box[9] = {0};
  long long max_polls = 0;
  int cap = 0;  // owned atoms the exported buffer holds (every rank)
  int natoms = 0;
  std::vector<int> gtype;  // global types (velocity draws at md_start)
  std::vector<Atom> own;
  std::vector<Ghost> ghosts;
  int nown = 0, nghost = 0;
  cudaStream_t stream = nullptr;
  DevArr<double> x, f, v, mass, minv, ev, part, ke;
  DevArr<int> type, origin;
  DevArr<double> shift;
  DevArr<Chain> chain;
  // MD
  bool md = false;
  b200dp_md_params mp{};
  ChainParams cp{};
  double dof = 0;
  long long step = 0, last_rebuild = 0;
  std::vector<double> x_at_rebuild;
  double max_move = 0;
  // NPT (isotropic): thermostat and barostat scalars on the host of every rank
  HostChain tch, pch;
  double omega_dot = 0, w_mass = 0, vol0 = 0, t_current = 0, vir_trace = 0;
  std::string err;
  ~b200dp_dd() {
    if (stream) {
      cudaStreamSynchronize(stream);
      cudaStreamDestroy(stream);
    }
  }
};

namespace {

b200dp_status dd_fail(b200dp_dd* dd, const std::string& msg, b200dp_status st = B200DP_ERR_CUDA) {
  dd->err = msg;
  return st;
}

// Device arrays of the current plan: owned + ghost positions and types, owned
// velocities and masses, the ghost origins and shifts (given to the engine).
b200dp_status upload_plan(b200dp_dd* dd) {
  const int n = dd->nown, g = dd->nghost, nall = n + g;
  if (n > dd->cap) return dd_fail(dd, "more owned atoms than the exported buffer holds", B200DP_ERR_CAPACITY);
  std::vector<double> x(3 * (size_t)nall), v(3 * (size_t)n), m(n), mi(n), sh(3 * (size_t)g);
  std::vector<int> t(nall), org(2 * (size_t)g);
  for (int i = 0; i < n; ++i) {
    const Atom& a = dd->own[i];
    for (int k = 0; k < 3; ++k) {
      x[3 * (size_t)i + k] = a.x[k];
      v[3 * (size_t)i + k] = a.v[k];
    }
    t[i] = a.type;
    m[i] = dd->md ? dd->mp.mass[a.type] : 1.0;
    mi[i] = 1.0 / m[i];
  }
  for (int j = 0; j < g; ++j) {
    const Ghost& q = dd->ghosts[j];
    for (int k = 0; k < 3; ++k) {
      x[3 * (size_t)(n + j) + k] = q.x[k];
      sh[3 * (size_t)j + k] = q.shift[k];
    }
    t[n + j] = q.type;
    org[2 * (size_t)j] = q.org_rank;
    org[2 * (size_t)j + 1] = q.org_row;
  }
  cudaError_t ce = cudaSuccess;
  auto chk = [&](cudaError_t e) {
    if (ce == cudaSuccess) ce = e;
  };
  chk(dd->x.ensure(3 * (size_t)nall));
  chk(dd->f.ensure(3 * (size_t)nall));
  chk(dd->type.ensure(nall));
  chk(dd->v.ensure(3 * (size_t)std::max(n, 1)));
  chk(dd->mass.ensure(std::max(n, 1)));
  chk(dd->minv.ensure(std::max(n, 1)));
  chk(dd->origin.ensure(2 * (size_t)std::max(g, 1)));
  chk(dd->shift.ensure(3 * (size_t)std::max(g, 1)));
  if (ce != cudaSuccess) return dd_fail(dd, "device allocation for the decomposed plan failed");
  cudaStream_t st = dd->stream;
  chk(cudaMemcpyAsync(dd->x.p, x.data(), sizeof(double) * x.size(), cudaMemcpyHostToDevice, st));
  chk(cudaMemcpyAsync(dd->type.p, t.data(), sizeof(int) * t.size(), cudaMemcpyHostToDevice, st));
  if (n) {
    chk(cudaMemcpyAsync(dd->v.p, v.data(), sizeof(double) * v.size(), cudaMemcpyHostToDevice, st));
    chk(cudaMemcpyAsync(dd->mass.p, m.data(), sizeof(double) * n, cudaMemcpyHostToDevice, st));
    chk(cudaMemcpyAsync(dd->minv.p, mi.data(), sizeof(double) * n, cudaMemcpyHostToDevice, st));
  }
  if (g) {
    chk(cudaMemcpyAsync(dd->origin.p, org.data(), sizeof(int) * org.size(), cudaMemcpyHostToDevice, st));
    chk(cudaMemcpyAsync(dd->shift.p, sh.data(), sizeof(double) * sh.size(), cudaMemcpyHostToDevice, st));
  }
  chk(cudaStreamSynchronize(st));
  if (ce != cudaSuccess) return dd_fail(dd, "uploading the decomposed plan failed");
  const b200dp_status rc = b200dp_fold_origins(dd->engine, g, dd->origin.p, dd->shift.p);
  if (rc != B200DP_OK) return dd_fail(dd, b200dp_last_error(dd->engine), rc);
  return B200DP_OK;
}

// Migration and a new ghost plan from the device positions and velocities
// (host synchronisation; every rank together).
b200dp_status rebuild(b200dp_dd* dd) {
  const int n = dd->nown;
  std::vector<double> x(3 * (size_t)n), v(3 * (size_t)n);
  if (n && (cudaMemcpyAsync(x.data(), dd->x.p, sizeof(double) * x.size(), cudaMemcpyDeviceToHost, dd->stream) !=
                cudaSuccess ||
            cudaMemcpyAsync(v.data(), dd->v.p, sizeof(double) * v.size(), cudaMemcpyDeviceToHost, dd->stream) !=
                cudaSuccess))
    return dd_fail(dd, "reading the owned atoms back failed");
  if (cudaStreamSynchronize(dd->stream) != cudaSuccess) return dd_fail(dd, "stream synchronisation failed");
  // the largest displacement since the last plan (the ghost shell must cover it)
  for (int i = 0; i < n; ++i) {
    double d2 = 0;
    for (int k = 0; k < 3; ++k) {
      const double dx = x[3 * (size_t)i + k] - dd->x_at_rebuild[3 * (size_t)i + k];
      d2 += dx * dx;
    }
    dd->max_move = std::max(dd->max_move, std::sqrt(d2));
  }
  for (int i = 0; i < n; ++i)
    for (int k = 0; k < 3; ++k) {
      dd->own[i].x[k] = x[3 * (size_t)i + k];
      dd->own[i].v[k] = v[3 * (size_t)i + k];
    }
  if (const char* e = migrate(*dd->comm, dd->dcmp, dd->own)) return dd_fail(dd, e);
  if (const char* e = build_halo(*dd->comm, dd->dcmp, dd->own, dd->ghosts)) return dd_fail(dd, e);
  dd->nown = (int)dd->own.size();
  dd->nghost = (int)dd->ghosts.size();
  dd->x_at_rebuild.resize(3 * (size_t)dd->nown);
  for (int i = 0; i < dd->nown; ++i)
    for (int k = 0; k < 3; ++k) dd->x_at_rebuild[3 * (size_t)i + k] = dd->own[i].x[k];
  return upload_plan(dd);
}

// The decomposed force call, enqueued on `st`.
b200dp_status force_call(b200dp_dd* dd, cudaStream_t st) {
  b200dp_engine* e = dd->engine;
  b200dp_status rc;
  if ((rc = b200dp_halo_publish(e, st, dd->nown, dd->x.p)) != B200DP_OK) return rc;
  if ((rc = b200dp_peer_reduce(e, st, 0, nullptr, nullptr, dd->max_polls)) != B200DP_OK) return rc;
  if ((rc = b200dp_halo_gather(e, st, dd->nown, dd->nghost, dd->x.p)) != B200DP_OK) return rc;
  if ((rc = b200dp_compute_device_fold(e, st, dd->nown, dd->nghost, dd->x.p, dd->type.p, dd->region, dd->ev.p,
                                       dd->f.p, dd->ev.p + 1)) != B200DP_OK)
    return rc;
  if ((rc = b200dp_peer_reduce(e, st, 10, dd->ev.p, dd->ev.p, dd->max_polls)) != B200DP_OK) return rc;
  return b200dp_fold_finish(e, st, dd->nown, dd->f.p);
}

// global kinetic energy (sum of m v^2 over all ranks) into ke[0]
b200dp_status global_mv2(b200dp_dd* dd, bool update_v, double dtf) {
  cudaStream_t st = dd->stream;
  count_launch();
  if (update_v)
    k_md_second<<<kRedBlocks, kMdThreads, 0, st>>>(dd->nown, dd->v.p, dd->f.p, dd->minv.p, dd->mass.p, dtf,
                                                   dd->part.p);
  else
    k_md_ke<<<kRedBlocks, kMdThreads, 0, st>>>(dd->nown, dd->v.p, dd->mass.p, dd->part.p);
  count_launch();
  k_dd_sum<<<1, 32, 0, st>>>(dd->part.p, kRedBlocks, dd->ke.p);
  return b200dp_peer_reduce(dd->engine, st, 1, dd->ke.p, dd->ke.p, dd->max_polls);
}

b200dp_status md_step(b200dp_dd* dd) {
  const double dt = dd->mp.dt, dtf = 0.5 * dt * kFtm2v;
  const bool nvt = dd->mp.ensemble == B200DP_MD_NVT;
  cudaStream_t st = dd->stream;
  const int grid = std::max(1, std::min(kRedBlocks * 4, (dd->nown + kMdThreads - 1) / kMdThreads));
  if (nvt) {
    count_launch();
    k_md_chain<<<1, 32, 0, st>>>(dd->cp, dd->chain.p, nullptr, 0, nullptr);
  }
  count_launch();
  k_md_first<<<grid, kMdThreads, 0, st>>>(dd->nown, dd->x.p, dd->v.p, dd->f.p, dd->minv.p,
                                          nvt ? dd->chain.p : nullptr, dtf, dt);
  ++dd->step;
  const int every = std::max(1, dd->mp.rebuild_every);
  if (dd->step - dd->last_rebuild >= every) {
    const b200dp_status rc = rebuild(dd);
    if (rc != B200DP_OK) return rc;
    dd->last_rebuild = dd->step;
  }
  b200dp_status rc = force_call(dd, st);
  if (rc != B200DP_OK) return rc;
  if ((rc = global_mv2(dd, true, dtf)) != B200DP_OK) return rc;
  if (nvt) {
    count_launch();
    k_md_chain<<<1, 32, 0, st>>>(dd->cp, dd->chain.p, dd->ke.p, 1, nullptr);
    count_launch();
    k_md_scale<<<grid, kMdThreads, 0, st>>>(dd->nown, dd->v.p, dd->chain.p);
  }
  return cudaGetLastError() == cudaSuccess ? B200DP_OK : B200DP_ERR_CUDA;
}

// One NPT step in LAMMPS' fix npt iso order (the order of the single-GPU
// driver, which keeps these scalars on the device): here the barostat and
// thermostat scalars live on the host of every rank, fed by the global
// kinetic energy and virial of the rendezvous (the same bits on every rank,
// so every rank computes the same box); one host read per step.
b200dp_status npt_step(b200dp_dd* dd) {
  const b200dp_md_params& p = dd->mp;
  const int n = dd->nown;
  const double natoms = (double)dd->natoms;
  const double dt = p.dt, dthalf = 0.5 * dt, dtf = 0.5 * dt * kFtm2v;
  const double kt = kBoltz * p.t_target, dof_boltz = dd->dof * kBoltz;
  const double ke_target = dof_boltz * p.t_target, p_hydro = p.p_target;
  cudaStream_t st = dd->stream;
  const int grid = std::max(1, std::min(kRedBlocks * 4, (n + kMdThreads - 1) / kMdThreads));
  auto omega_force = [&](double t_cur, double vir_tr) {
    const double vol = dd->box[0] * dd->box[4] * dd->box[8];
    const double p_cur = (dof_boltz * t_cur + vir_tr) / (3.0 * vol) * kNktv2p;
    const double mtk1 = dof_boltz * t_cur / (3.0 * natoms);
    dd->omega_dot += ((p_cur - p_hydro) * vol / (dd->w_mass * kNktv2p) + mtk1 / dd->w_mass) * dthalf;
  };
  // ---- initial half
  dd->pch.barostat(dd->omega_dot, dd->w_mass, kt, dt);
  const double s_t = dd->tch.thermostat(dd->t_current, dof_boltz, ke_target, kt, dt);
  omega_force(dd->t_current, dd->vir_trace);
  const double mtk2 = 3.0 * dd->omega_dot / (3.0 * natoms);
  const double fp = std::exp(-0.25 * dt * (dd->omega_dot + mtk2));
  const double e = std::exp(dthalf * dd->omega_dot);
  count_launch();
  k_npt_first<<<grid, kMdThreads, 0, st>>>(n, dd->x.p, dd->v.p, dd->f.p, dd->minv.p, s_t * fp * fp, dtf, dt, e);
  const double r = e * e;
  for (int d = 0; d < 3; ++d) dd->box[4 * d] *= r;
  dd->dcmp.scale(r);
  for (int d = 0; d < 3; ++d) {
    dd->region[d] = dd->dcmp.lo[d] - dd->dcmp.halo;
    dd->region[3 + d] = dd->dcmp.hi[d] + dd->dcmp.halo;
  }
  ++dd->step;
  b200dp_status rc;
  const int every = std::max(1, p.rebuild_every);
  if (dd->step - dd->last_rebuild >= every) {
    if ((rc = rebuild(dd)) != B200DP_OK) return rc;
    dd->last_rebuild = dd->step;
  } else {
    const double ratio[3] = {r, r, r};
    if ((rc = b200dp_fold_scale_shifts(dd->engine, st, ratio)) != B200DP_OK) return rc;
  }
  if ((rc = force_call(dd, st)) != B200DP_OK) return rc;
  // ---- final half, over the atoms owned after the rebuild (migration changes the count)
  const int n2 = dd->nown;
  const int grid2 = std::max(1, std::min(kRedBlocks * 4, (n2 + kMdThreads - 1) / kMdThreads));
  count_launch();
  k_npt_second<<<kRedBlocks, kMdThreads, 0, st>>>(n2, dd->v.p, dd->f.p, dd->minv.p, dd->mass.p, dtf, fp * fp,
                                                  dd->part.p);
  count_launch();
  k_dd_sum<<<1, 32, 0, st>>>(dd->part.p, kRedBlocks, dd->ke.p);
  if ((rc = b200dp_peer_reduce(dd->engine, st, 1, dd->ke.p, dd->ke.p, dd->max_polls)) != B200DP_OK) return rc;
  double mv2 = 0, ev[10];
  if (cudaMemcpyAsync(&mv2, dd->ke.p, sizeof(double), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(ev, dd->ev.p, sizeof(ev), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return dd_fail(dd, "reading the global kinetic energy and virial failed");
  dd->t_current = mv2 * kMvv2e / dof_boltz;
  dd->vir_trace = ev[1] + ev[5] + ev[9];
  omega_force(dd->t_current, dd->vir_trace);
  const double s_t2 = dd->tch.thermostat(dd->t_current, dof_boltz, ke_target, kt, dt);
  count_launch();
  k_md_scale_by<<<grid2, kMdThreads, 0, st>>>(n2, dd->v.p, s_t2);
  dd->pch.barostat(dd->omega_dot, dd->w_mass, kt, dt);
  return cudaGetLastError() == cudaSuccess ? B200DP_OK : B200DP_ERR_CUDA;
}

}  // namespace

extern "C" {

b200dp_status b200dp_dd_unique_id(void* id) {
  if (!id) return B200DP_ERR_INVALID;
  ncclUniqueId u;
  if (ncclGetUniqueId(&u) != ncclSuccess) return B200DP_ERR_CUDA;
  static_assert(sizeof(u) == 128, "NCCL unique id size");
  std::memcpy(id, &u, sizeof(u));
  return B200DP_OK;
}

void b200dp_dd_params_default(b200dp_dd_params* p) {
  if (!p) return;
  std::memset(p, 0, sizeof(*p));
  p->grid[0] = p->grid[1] = p->grid[2] = 1;
  p->halo = 8.0;
}

b200dp_status b200dp_dd_create(b200dp_engine* engine, const void* id, int nranks, int rank, const double* box,
                               const b200dp_dd_params* p, int natoms, const double* coord, const int* atype,
                               b200dp_dd** out) {
  if (!engine || !id || nranks < 1 || rank < 0 || rank >= nranks || !box || !p || natoms < 0 || !out ||
      (natoms > 0 && (!coord || !atype)) || p->grid[0] * p->grid[1] * p->grid[2] != nranks)
    return B200DP_ERR_INVALID;
  *out = nullptr;
  auto dd = std::make_unique<b200dp_dd>();
  dd->engine = engine;
  if (dd->dcmp.init(box, p->grid, rank, p->halo)) return B200DP_ERR_INVALID;  // orthorhombic, halo <= sub-box
  b200dp_model_info info;
  if (b200dp_model_info_get(engine, &info) != B200DP_OK || p->halo < info.rcut) return B200DP_ERR_INVALID;
  std::memcpy(dd->box, box, sizeof(dd->box));
  dd->device = b200dp_engine_device(engine);
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  if (cudaStreamCreateWithFlags(&dd->stream, cudaStreamNonBlocking) != cudaSuccess) return B200DP_ERR_CUDA;
  dd->max_polls = p->max_polls;
  dd->natoms = natoms;
  dd->gtype.assign(atype, atype + natoms);
  for (int d = 0; d < 3; ++d) {
    dd->region[d] = dd->dcmp.lo[d] - dd->dcmp.halo;
    dd->region[3 + d] = dd->dcmp.hi[d] + dd->dcmp.halo;
  }
  // NCCL communicator (collective over the ranks)
  auto c = std::make_unique<NcclComm>();
  c->rank = rank;
  c->size = nranks;
  c->st = dd->stream;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  if (ncclCommInitRank(&c->comm, nranks, u, rank) != ncclSuccess) return B200DP_ERR_CUDA;
  dd->comm = std::move(c);
  // owned atoms: those whose wrapped position lies in this rank's sub-box
  for (int i = 0; i < natoms; ++i) {
    Atom a;
    std::memset(&a, 0, sizeof(a));
    for (int k = 0; k < 3; ++k) a.x[k] = wrap1(coord[3 * (size_t)i + k], dd->dcmp.L[k]);
    if (!dd->dcmp.owns(a.x)) continue;
    a.id = i;
    a.type = atype[i];
    dd->own.push_back(a);
  }
  // one capacity for every rank's exported buffer
  int mine = (int)dd->own.size();
  std::vector<int> counts(nranks);
  if (!dd->comm->allgather(&mine, sizeof(int), counts.data())) return B200DP_ERR_CUDA;
  const int mx = *std::max_element(counts.begin(), counts.end());
  dd->cap = std::max(p->capacity, mx + mx / 2 + 1024);
  unsigned char handle[64];
  b200dp_status rc = b200dp_fold_export(engine, dd->cap, handle);
  if (rc != B200DP_OK) return rc;
  std::vector<unsigned char> handles(64 * (size_t)nranks);
  if (!dd->comm->allgather(handle, 64, handles.data())) return B200DP_ERR_CUDA;
  if ((rc = b200dp_fold_connect(engine, nranks, rank, handles.data())) != B200DP_OK) return rc;
  if (build_halo(*dd->comm, dd->dcmp, dd->own, dd->ghosts)) return B200DP_ERR_CUDA;
  dd->nown = (int)dd->own.size();
  dd->nghost = (int)dd->ghosts.size();
  cudaError_t ce = cudaSuccess;
  auto chk = [&](cudaError_t e) {
    if (ce == cudaSuccess) ce = e;
  };
  chk(dd->ev.ensure(10));
  chk(dd->part.ensure(kRedBlocks));
  chk(dd->ke.ensure(1));
  chk(dd->chain.ensure(1));
  if (ce != cudaSuccess) return B200DP_ERR_CUDA;
  dd->x_at_rebuild.resize(3 * (size_t)dd->nown);
  for (int i = 0; i < dd->nown; ++i)
    for (int k = 0; k < 3; ++k) dd->x_at_rebuild[3 * (size_t)i + k] = dd->own[i].x[k];
  if ((rc = upload_plan(dd.get())) != B200DP_OK) return rc;
  *out = dd.release();
  return B200DP_OK;
}

void b200dp_dd_destroy(b200dp_dd* dd) {
  if (!dd) return;
  cudaSetDevice(dd->device);
  delete dd;
}

const char* b200dp_dd_last_error(const b200dp_dd* dd) { return dd ? dd->err.c_str() : "null handle"; }

void* b200dp_dd_stream(b200dp_dd* dd) { return dd ? dd->stream : nullptr; }

b200dp_status b200dp_dd_counts(b200dp_dd* dd, int* nowned, int* nghost) {
  if (!dd) return B200DP_ERR_INVALID;
  if (nowned) *nowned = dd->nown;
  if (nghost) *nghost = dd->nghost;
  return B200DP_OK;
}

b200dp_status b200dp_dd_force(b200dp_dd* dd, void* stream) {
  if (!dd) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  return force_call(dd, stream ? static_cast<cudaStream_t>(stream) : dd->stream);
}

b200dp_status b200dp_dd_result(b200dp_dd* dd, void* stream, double* energy, double* virial) {
  if (!dd) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : dd->stream;
  double ev[10];
  if (cudaMemcpyAsync(ev, dd->ev.p, sizeof(ev), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return dd_fail(dd, "reading energy and virial failed");
  const b200dp_status rc = b200dp_check(dd->engine);
  if (rc != B200DP_OK) return dd_fail(dd, b200dp_last_error(dd->engine), rc);
  if (energy) *energy = ev[0];
  if (virial) std::memcpy(virial, ev + 1, sizeof(double) * 9);
  return B200DP_OK;
}

b200dp_status b200dp_dd_owned(b200dp_dd* dd, long long* ids, double* coord, double* vel, double* force) {
  if (!dd) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  const size_t b = sizeof(double) * 3 * (size_t)dd->nown;
  cudaStream_t st = dd->stream;
  if (dd->nown && ((coord && cudaMemcpyAsync(coord, dd->x.p, b, cudaMemcpyDeviceToHost, st) != cudaSuccess) ||
                   (vel && cudaMemcpyAsync(vel, dd->v.p, b, cudaMemcpyDeviceToHost, st) != cudaSuccess) ||
                   (force && cudaMemcpyAsync(force, dd->f.p, b, cudaMemcpyDeviceToHost, st) != cudaSuccess)))
    return dd_fail(dd, "reading the owned atoms failed");
  if (cudaStreamSynchronize(st) != cudaSuccess) return dd_fail(dd, "stream synchronisation failed");
  if (ids)
    for (int i = 0; i < dd->nown; ++i) ids[i] = dd->own[i].id;
  return B200DP_OK;
}

b200dp_status b200dp_dd_set_positions(b200dp_dd* dd, void* stream, const double* coord) {
  if (!dd || (dd->nown && !coord)) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : dd->stream;
  if (dd->nown &&
      cudaMemcpyAsync(dd->x.p, coord, sizeof(double) * 3 * (size_t)dd->nown, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return dd_fail(dd, "copying positions failed");
  return B200DP_OK;
}

b200dp_status b200dp_dd_get_forces(b200dp_dd* dd, void* stream, double* force, double* ev) {
  if (!dd) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : dd->stream;
  if (force && dd->nown &&
      cudaMemcpyAsync(force, dd->f.p, sizeof(double) * 3 * (size_t)dd->nown, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return dd_fail(dd, "copying forces failed");
  if (ev && cudaMemcpyAsync(ev, dd->ev.p, sizeof(double) * 10, cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return dd_fail(dd, "copying energy and virial failed");
  return B200DP_OK;
}

b200dp_status b200dp_dd_md_start(b200dp_dd* dd, const b200dp_md_params* params, const double* vel) {
  if (!dd || !params) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  const b200dp_md_params& p = *params;
  if (!(p.dt > 0) || (p.ensemble != B200DP_MD_NVE && p.ensemble != B200DP_MD_NVT && p.ensemble != B200DP_MD_NPT))
    return B200DP_ERR_INVALID;
  if (p.ensemble != B200DP_MD_NVE && (p.chain < 1 || p.chain > kMaxChain || !(p.t_target > 0) || !(p.t_damp > 0)))
    return B200DP_ERR_INVALID;
  if (p.ensemble == B200DP_MD_NPT && (p.pchain < 1 || p.pchain > kMaxChain || !(p.p_damp > 0)))
    return B200DP_ERR_INVALID;  // the box is orthorhombic (checked at creation); isotropic barostat
  if (!vel && !(p.t_init > 0)) return B200DP_ERR_INVALID;
  const int natoms = dd->natoms;
  std::vector<double> mass(natoms);
  for (int i = 0; i < natoms; ++i) {
    const int t = dd->gtype[i];
    if (t < 0 || t >= 8 || !(p.mass[t] > 0)) return B200DP_ERR_BAD_TYPE;
    mass[i] = p.mass[t];
  }
  dd->mp = p;
  dd->md = true;
  dd->dof = 3.0 * natoms - 3.0;
  // the global velocities (given, or the seeded draw every rank makes alike)
  std::vector<double> v(3 * (size_t)natoms);
  if (vel)
    std::copy(vel, vel + 3 * (size_t)natoms, v.begin());
  else
    init_velocities(natoms, mass.data(), p.t_init, p.seed, dd->dof, v.data());
  double mv2 = 0;
  for (int i = 0; i < natoms; ++i)
    for (int c = 0; c < 3; ++c) mv2 += mass[i] * v[3 * (size_t)i + c] * v[3 * (size_t)i + c];
  for (Atom& a : dd->own)
    for (int c = 0; c < 3; ++c) a.v[c] = v[3 * (size_t)a.id + c];
  // chain parameters and state (as the single-GPU driver)
  Chain ch;
  std::memset(&ch, 0, sizeof(ch));
  ch.factor = 1.0;
  ch.t_current = mv2 * kMvv2e / (dd->dof * kBoltz);
  ChainParams& cp = dd->cp;
  std::memset(&cp, 0, sizeof(cp));
  if (p.ensemble != B200DP_MD_NVE) {
    const double w = 1.0 / p.t_damp;
    cp.M = p.chain;
    cp.dof_boltz = dd->dof * kBoltz;
    cp.ke_target = dd->dof * kBoltz * p.t_target;
    cp.boltz_t = kBoltz * p.t_target;
    cp.dt4 = 0.25 * p.dt;
    cp.dt8 = 0.125 * p.dt;
    cp.dthalf = 0.5 * p.dt;
    cp.mass[0] = cp.ke_target / (w * w);
    for (int i = 1; i < cp.M; ++i) cp.mass[i] = cp.boltz_t / (w * w);
    for (int i = 1; i < cp.M; ++i)
      ch.eta_dotdot[i] = (cp.mass[i - 1] * ch.eta_dot[i - 1] * ch.eta_dot[i - 1] - cp.boltz_t) / cp.mass[i];
  }
  if (cudaMemcpy(dd->chain.p, &ch, sizeof(ch), cudaMemcpyHostToDevice) != cudaSuccess)
    return dd_fail(dd, "uploading the chain failed");
  b200dp_status rc = upload_plan(dd);  // velocities and masses of the owned atoms
  if (rc != B200DP_OK) return rc;
  dd->step = dd->last_rebuild = 0;
  dd->max_move = 0;
  // forces and kinetic energy of the initial configuration
  if ((rc = force_call(dd, dd->stream)) != B200DP_OK) return rc;
  if ((rc = global_mv2(dd, false, 0.0)) != B200DP_OK) return rc;
  if (p.ensemble == B200DP_MD_NPT) {
    const double wp = 1.0 / p.p_damp, kt = kBoltz * p.t_target;
    dd->tch = HostChain();
    dd->pch = HostChain();
    dd->tch.init(p.chain, cp.mass[0], p.chain > 1 ? cp.mass[1] : 0.0, cp.boltz_t);
    dd->pch.init(p.pchain, kt / (wp * wp), kt / (wp * wp), kt);
    dd->w_mass = (natoms + 1) * kt / (wp * wp);
    dd->vol0 = dd->box[0] * dd->box[4] * dd->box[8];
    dd->omega_dot = 0;
    dd->t_current = ch.t_current;
    double ev[10];
    if (cudaMemcpyAsync(ev, dd->ev.p, sizeof(ev), cudaMemcpyDeviceToHost, dd->stream) != cudaSuccess ||
        cudaStreamSynchronize(dd->stream) != cudaSuccess)
      return B200DP_ERR_CUDA;
    dd->vir_trace = ev[1] + ev[5] + ev[9];
  }
  return cudaStreamSynchronize(dd->stream) == cudaSuccess ? B200DP_OK : B200DP_ERR_CUDA;
}

b200dp_status b200dp_dd_md_run(b200dp_dd* dd, int nsteps) {
  if (!dd || !dd->md || nsteps < 0) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  for (int s = 0; s < nsteps; ++s) {
    const b200dp_status rc = dd->mp.ensemble == B200DP_MD_NPT ? npt_step(dd) : md_step(dd);
    if (rc != B200DP_OK) return rc;
  }
  return B200DP_OK;
}

b200dp_status b200dp_dd_md_thermo(b200dp_dd* dd, double* thermo) {
  if (!dd || !dd->md || !thermo) return B200DP_ERR_INVALID;
  if (cudaSetDevice(dd->device) != cudaSuccess) return B200DP_ERR_CUDA;
  double ev[10], mv2 = 0;
  Chain ch;
  cudaStream_t st = dd->stream;
  if (cudaMemcpyAsync(ev, dd->ev.p, sizeof(ev), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(&mv2, dd->ke.p, sizeof(double), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaMemcpyAsync(&ch, dd->chain.p, sizeof(ch), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return dd_fail(dd, "reading the thermodynamic state failed");
  const b200dp_status rc = b200dp_check(dd->engine);
  if (rc != B200DP_OK) return dd_fail(dd, b200dp_last_error(dd->engine), rc);
  b200dp_model_info info;
  b200dp_model_info_get(dd->engine, &info);
  if (dd->max_move > 0.5 * (dd->dcmp.halo - info.rcut))
    return dd_fail(dd, "an atom moved more than (halo - rcut) / 2 between ghost plans: rebuild more often",
                   B200DP_ERR_CAPACITY);
  const bool nvt = dd->mp.ensemble == B200DP_MD_NVT, npt = dd->mp.ensemble == B200DP_MD_NPT;
  // kinetic energy: after the chain's rescaling the chain's temperature (NVT: device state, NPT:
  // the host scalars), else the reduced sum
  const double temp = nvt ? ch.t_current : npt ? dd->t_current : mv2 * kMvv2e / (dd->dof * kBoltz);
  const double ke = 0.5 * dd->dof * kBoltz * temp;
  double e_chain = 0;
  const double vol = dd->box[0] * dd->box[4] * dd->box[8];
  if (npt) {
    const double kt = kBoltz * dd->mp.t_target;
    e_chain = dd->tch.energy(dd->cp.ke_target, kt) + dd->pch.energy(kt, kt) +
              1.5 * dd->w_mass * dd->omega_dot * dd->omega_dot + dd->mp.p_target * (vol - dd->vol0) / kNktv2p;
  } else if (nvt) {
    const ChainParams& cp = dd->cp;
    e_chain = cp.ke_target * ch.eta[0];
    for (int i = 1; i < cp.M; ++i) e_chain += cp.boltz_t * ch.eta[i];
    for (int i = 0; i < cp.M; ++i) e_chain += 0.5 * cp.mass[i] * ch.eta_dot[i] * ch.eta_dot[i];
  }
  thermo[0] = (double)dd->step;
  thermo[1] = ev[0];
  thermo[2] = ke;
  thermo[3] = temp;
  thermo[4] = ev[0] + ke + e_chain;
  thermo[5] = (dd->dof * kBoltz * temp + ev[1] + ev[5] + ev[9]) / (3.0 * vol) * kNktv2p;
  thermo[6] = vol;
  thermo[7] = e_chain;
  return B200DP_OK;
}

// CPU check of the host plan: nranks threads stand in for the ranks.
b200dp_status b200dp_dd_plan_emulate(int nranks, const int* grid, const double* box, double halo, int natoms,
                                     const double* coord, const double* disp, long long* owned_ids,
                                     int* owned_count, long long* ghost_ids, double* ghost_x, double* ghost_shift,
                                     int* ghost_origin, int* ghost_count, int ghost_cap) {
  if (nranks < 1 || !grid || grid[0] * grid[1] * grid[2] != nranks || !box || natoms < 0 || (natoms && !coord) ||
      !owned_ids || !owned_count || !ghost_count || ghost_cap < 0)
    return B200DP_ERR_INVALID;
  Mailboxes mb;
  mb.n = nranks;
  mb.q.resize((size_t)nranks * nranks);
  std::vector<std::vector<Atom>> own(nranks);
  std::vector<std::vector<Ghost>> gh(nranks);
  std::vector<std::string> errs(nranks);
  std::vector<std::thread> th;
  for (int r = 0; r < nranks; ++r) {
    th.emplace_back([&, r] {
      ThreadComm c;
      c.rank = r;
      c.size = nranks;
      c.mb = &mb;
      Decomp d;
      if (const char* e = d.init(box, grid, r, halo)) {
        errs[r] = e;
        return;
      }
      for (int i = 0; i < natoms; ++i) {
        Atom a;
        std::memset(&a, 0, sizeof(a));
        for (int k = 0; k < 3; ++k) a.x[k] = wrap1(coord[3 * (size_t)i + k], d.L[k]);
        if (!d.owns(a.x)) continue;
        a.id = i;
        own[r].push_back(a);
      }
      if (disp) {  // positions after a move, then the migration to the new owners
        for (Atom& a : own[r])
          for (int k = 0; k < 3; ++k) a.x[k] += disp[3 * (size_t)a.id + k];
        if (const char* e = migrate(c, d, own[r])) {
          errs[r] = e;
          return;
        }
      }
      if (const char* e = build_halo(c, d, own[r], gh[r])) errs[r] = e;
    });
  }
  for (auto& t : th) t.join();
  for (int r = 0; r < nranks; ++r)
    if (!errs[r].empty()) return B200DP_ERR_INVALID;
  size_t o = 0, g = 0;
  for (int r = 0; r < nranks; ++r) {
    owned_count[r] = (int)own[r].size();
    for (const Atom& a : own[r]) owned_ids[o++] = a.id;
    ghost_count[r] = (int)gh[r].size();
    for (const Ghost& q : gh[r]) {
      if (g < (size_t)ghost_cap) {
        if (ghost_ids) ghost_ids[g] = q.id;
        for (int k = 0; k < 3; ++k) {
          if (ghost_x) ghost_x[3 * g + k] = q.x[k];
          if (ghost_shift) ghost_shift[3 * g + k] = q.shift[k];
        }
        if (ghost_origin) {
          ghost_origin[2 * g] = q.org_rank;
          ghost_origin[2 * g + 1] = q.org_row;
        }
      }
      ++g;
    }
  }
  return g <= (size_t)ghost_cap ? B200DP_OK : B200DP_ERR_CAPACITY;
}

}  // extern "C"
