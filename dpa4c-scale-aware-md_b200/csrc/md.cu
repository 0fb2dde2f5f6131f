// Molecular-dynamics driver around the force engine: velocity Verlet with an
// optional Nose-Hoover chain thermostat (NVT) or thermostat + isotropic MTK
// barostat (NPT), state resident on the device.
//
// Semantics follow LAMMPS `fix nve` / `fix nvt` in metal units (the reference
// drives its force call from LAMMPS' Kokkos Verlet with `fix nh`,
// components/lammps/overlays/src/KOKKOS/fix_nh_kokkos.cpp:863-1001, and keeps
// the chain recurrence on the device,
// components/lammps/overlays/src/KOKKOS/dpa_fast_step_kokkos.h:307-400):
//   initial half: [NVT] chain update from the current temperature, v *= s;
//                 v += dt/2 F/m; x += dt v
//   force call (b200dp_compute_device, periodic box)
//   final half:   v += dt/2 F/m; temperature; [NVT] chain update, v *= s
// The chain follows the Martyna-Tuckerman-Klein integration of LAMMPS' FixNH
// (one Suzuki-Yoshida stage, chain length M, masses Q0 = dof kB T0 / w^2,
// Qi = kB T0 / w^2 with w = 1 / t_damp).  Every step is enqueued on one stream
// with no host synchronisation; reductions use a fixed grid and order, so a
// trajectory is bitwise reproducible.
//
// NPT follows LAMMPS' fix npt iso with the MTK terms (FixNH: nhc_press_integrate,
// nhc_temp_integrate, nh_omega_dot, nh_v_press, remap):
//   initial: barostat chain; thermostat chain (v *= s); pressure from the last
//            virial; omega_dot += dt/2 F_omega; v *= exp(-dt/2 (omega_dot + mtk2));
//            v += dt/2 F/m; x *= exp(dt omega_dot) around the drift x += dt v
//            (two half remaps), box scaled the same way
//   force call in the new box
//   final:   v += dt/2 F/m; v *= exp(-dt/2 (omega_dot + mtk2)); temperature and
//            pressure; omega_dot += dt/2 F_omega; thermostat chain; barostat chain
// The scalar chains and the box live on the device too (NptState, advanced by
// one-thread kernels), and the force call reads the box from device memory
// (b200dp_compute_device_dbox), so an NPT step needs no host round trip and
// whole neighbour cycles replay as CUDA graphs, as for NVT.  The host reads the
// state back only at its synchronisation points (thermo, snapshot, restore),
// where it also re-references the binning grid when the box has drifted more
// than 5 % from the box the grid was built for (the grid serves boxes down to
// 90 % of it; a step that goes lower sets a flag reported as an error).  The
// box is scaled about the origin (LAMMPS scales about the box centre; the two
// differ by a uniform translation).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/b200dp.h"
#include "common.cuh"

namespace b200dp {
namespace {

#include "md_kernels.cuh"

// Device state of the NPT integrator: the two chains, the barostat scalars,
// the box and the step's velocity / position factors.
struct NptState {
  HostChain tch, pch;
  double omega_dot, w_mass, vol0, t_current, vir_trace, epot;
  double box[9];
  double sv1, e, fp2, s_t2;
  int box_low;  // the box fell below the range the binning grid serves
};
struct NptParams {
  double dt, kt, dof_boltz, ke_target, p_hydro, natoms;
  double min_box[3];
};

__device__ void npt_omega_force(const NptParams& p, NptState* s, double t_cur, double vir_tr) {
  const double vol = s->box[0] * s->box[4] * s->box[8];
  const double p_cur = (p.dof_boltz * t_cur + vir_tr) / (3.0 * vol) * kNktv2p;
  const double mtk1 = p.dof_boltz * t_cur / (3.0 * p.natoms);
  s->omega_dot += ((p_cur - p.p_hydro) * vol / (s->w_mass * kNktv2p) + mtk1 / s->w_mass) * (0.5 * p.dt);
}

// Initial half of an NPT step: barostat chain, thermostat chain, the barostat
// force, the velocity / remap factors and the new box.
__global__ void k_npt_pre(NptParams p, NptState* __restrict__ s) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  s->pch.barostat(s->omega_dot, s->w_mass, p.kt, p.dt);
  const double s_t = s->tch.thermostat(s->t_current, p.dof_boltz, p.ke_target, p.kt, p.dt);
  npt_omega_force(p, s, s->t_current, s->vir_trace);
  const double mtk2 = 3.0 * s->omega_dot / (3.0 * p.natoms);
  const double fp = exp(-0.25 * p.dt * (s->omega_dot + mtk2));
  const double e = exp(0.5 * p.dt * s->omega_dot);
  s->sv1 = s_t * fp * fp;
  s->e = e;
  s->fp2 = fp * fp;
  for (int d = 0; d < 3; ++d) {
    s->box[4 * d] *= e * e;
    if (s->box[4 * d] < p.min_box[d]) s->box_low = 1;
  }
}

// k_npt_first / k_npt_second with their factors from the device state.
__global__ void k_npt_first_dev(int n, double* __restrict__ x, double* __restrict__ v, const double* __restrict__ f,
                                const double* __restrict__ minv, const NptState* __restrict__ s, double dtf,
                                double dt) {
  const double sv = s->sv1, e = s->e;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double w = dtf * minv[i];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double vv = v[3 * i + c] * sv + w * f[3 * i + c];
      v[3 * i + c] = vv;
      x[3 * i + c] = e * (e * x[3 * i + c] + dt * vv);
    }
  }
}

__global__ void __launch_bounds__(kMdThreads) k_npt_second_dev(int n, double* __restrict__ v,
                                                               const double* __restrict__ f,
                                                               const double* __restrict__ minv,
                                                               const double* __restrict__ mass, double dtf,
                                                               const NptState* __restrict__ s,
                                                               double* __restrict__ part) {
  __shared__ double sh[kMdThreads / 32];
  const double sv = s->fp2;
  double acc = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double w = dtf * minv[i];
    double s2 = 0.0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double vv = (v[3 * i + c] + w * f[3 * i + c]) * sv;
      v[3 * i + c] = vv;
      s2 += vv * vv;
    }
    acc += mass[i] * s2;
  }
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int w = 0; w < kMdThreads / 32; ++w) b += sh[w];
    part[blockIdx.x] = b;
  }
}

// Final half: temperature from the kinetic-energy partials, the virial's trace,
// the barostat force, the thermostat (its factor applied by k_npt_scale) and
// the barostat chain.  One warp.
__global__ void k_npt_post(NptParams p, NptState* __restrict__ s, const double* __restrict__ part, int nparts,
                           const double* __restrict__ vir, const double* __restrict__ epot) {
  const double mv2 = sum_parts(part, nparts);
  if (threadIdx.x != 0) return;
  s->t_current = mv2 * kMvv2e / p.dof_boltz;
  s->vir_trace = vir[0] + vir[4] + vir[8];
  s->epot = epot[0];
  npt_omega_force(p, s, s->t_current, s->vir_trace);
  s->s_t2 = s->tch.thermostat(s->t_current, p.dof_boltz, p.ke_target, p.kt, p.dt);
  s->pch.barostat(s->omega_dot, s->w_mass, p.kt, p.dt);
}

__global__ void k_npt_scale(int n, double* __restrict__ v, const NptState* __restrict__ s) {
  const double f = s->s_t2;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * n; i += gridDim.x * blockDim.x) v[i] *= f;
}

template <class T>
struct Dev {
  T* p = nullptr;
  cudaError_t alloc(size_t n) { return cudaMalloc(&p, sizeof(T) * std::max<size_t>(n, 1)); }
  ~Dev() {
    if (p) cudaFree(p);
  }
};

}  // namespace
}  // namespace b200dp

using namespace b200dp;

namespace b200dp {
namespace {
// Restart snapshot: this header (host scalars of the integrator), then the
// device state, each section 256-byte aligned.  Device-resident snapshots
// are taken on the MD stream without a host round trip; a restart file is the
// same byte image.
struct SnapHeader {
  char magic[8];
  int n, ensemble;
  long long step;
  double box[9], volume, dof;
  HostChain tch, pch;
  ChainParams cp;
  double omega_dot, w_mass, vol0, t_current, vir_trace, epot;
  double dt;
  unsigned long long bytes;
};
constexpr char kSnapMagic[8] = {'B', '2', 'D', 'P', 'M', 'D', 'S', '2'};
constexpr size_t snap_align(size_t b) { return (b + 255) & ~(size_t)255; }
struct SnapLayout {
  size_t x, v, f, e, vir, part, chain, npt, total;
  explicit SnapLayout(int n) {
    const size_t n3 = sizeof(double) * 3 * (size_t)n;
    x = snap_align(sizeof(SnapHeader));
    v = x + snap_align(n3);
    f = v + snap_align(n3);
    e = f + snap_align(n3);
    vir = e + snap_align(sizeof(double));
    part = vir + snap_align(9 * sizeof(double));
    chain = part + snap_align(kRedBlocks * sizeof(double));
    npt = chain + snap_align(sizeof(Chain));
    total = npt + snap_align(sizeof(NptState));
  }
};
}  // namespace
}  // namespace b200dp

struct b200dp_md {
  b200dp_engine* engine = nullptr;
  b200dp_md_params p{};
  int n = 0, ensemble = 0;
  double box[9] = {0}, volume = 0, dof = 0;
  long long step = 0;
  cudaStream_t stream = nullptr;
  Dev<double> x, v, f, minv, mass, e, vir, part, ke;
  Dev<int> atype;
  Dev<Chain> chain;
  ChainParams cp{};
  // NPT: host copies of the device state (refreshed at the synchronisation
  // points) and the reference box of the binning grid
  HostChain tch, pch;
  double omega_dot = 0, w_mass = 0, vol0 = 0, t_current = 0, vir_trace = 0, epot = 0;
  Dev<NptState> npt;
  double box_ref[9] = {0};
  std::string err;
  SnapHeader snap_stage{};
  // one neighbour-rebuild cycle of steps recorded as a CUDA graph and replayed
  // (every step's work is enqueued with no host decision left, the skin check
  // and rebuild being gated on the device, the NPT scalars advanced there)
  cudaGraphExec_t cycle = nullptr;
  int cycle_len = 0;
  bool cycle_failed = false;
};

namespace {
constexpr double kGridMinScale = 0.9;   // the grid serves boxes down to this fraction of the reference
constexpr double kGridReref = 0.05;     // re-reference when the box drifted this much (relative)

NptParams npt_params(const b200dp_md* md) {
  NptParams q;
  q.dt = md->p.dt;
  q.kt = kBoltz * md->p.t_target;
  q.dof_boltz = md->dof * kBoltz;
  q.ke_target = q.dof_boltz * md->p.t_target;
  q.p_hydro = md->p.p_target;
  q.natoms = (double)md->n;
  for (int d = 0; d < 3; ++d) q.min_box[d] = kGridMinScale * md->box_ref[4 * d];
  return q;
}
double* npt_box(b200dp_md* md) { return reinterpret_cast<double*>(reinterpret_cast<char*>(md->npt.p) + offsetof(NptState, box)); }

// Host copies of the device NPT state (the caller synchronised the stream); a
// box that drifted from the grid's reference re-references the grid (and drops
// the recorded cycle, whose calls carry the old grid).
b200dp_status npt_refresh(b200dp_md* md) {
  NptState h;
  if (cudaMemcpyAsync(&h, md->npt.p, sizeof(h), cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
      cudaStreamSynchronize(md->stream) != cudaSuccess)
    return B200DP_ERR_CUDA;
  md->tch = h.tch;
  md->pch = h.pch;
  md->omega_dot = h.omega_dot;
  md->w_mass = h.w_mass;
  md->vol0 = h.vol0;
  md->t_current = h.t_current;
  md->vir_trace = h.vir_trace;
  md->epot = h.epot;
  std::memcpy(md->box, h.box, sizeof(md->box));
  md->volume = md->box[0] * md->box[4] * md->box[8];
  if (h.box_low) {
    md->err = "the box shrank below the range of the binning grid within one run call";
    return B200DP_ERR_CAPACITY;
  }
  bool reref = false;
  for (int d = 0; d < 3; ++d)
    reref = reref || std::fabs(md->box[4 * d] / md->box_ref[4 * d] - 1.0) > kGridReref;
  if (reref) {
    std::memcpy(md->box_ref, md->box, sizeof(md->box_ref));
    if (md->cycle) cudaGraphExecDestroy(md->cycle);
    md->cycle = nullptr;
    md->cycle_failed = false;
  }
  return B200DP_OK;
}
}  // namespace

extern "C" {

b200dp_status b200dp_md_params_default(b200dp_md_params* p) {
  if (!p) return B200DP_ERR_INVALID;
  std::memset(p, 0, sizeof(*p));
  p->dt = 0.0005;  // 0.5 fs
  p->ensemble = B200DP_MD_NVE;
  p->chain = 3;
  p->t_target = 300.0;
  p->t_damp = 0.05;  // 100 steps of 0.5 fs
  p->p_target = 1.0;
  p->p_damp = 0.5;
  p->pchain = 3;
  p->rebuild_every = 10;
  p->skin = 2.0;
  return B200DP_OK;
}

b200dp_status b200dp_md_create(b200dp_engine* engine, int natoms, const double* coord, const double* vel,
                               const int* atype, const double* box, const b200dp_md_params* params,
                               b200dp_md** out) {
  if (!engine || !out || natoms <= 0 || !coord || !atype || !box || !params) return B200DP_ERR_INVALID;
  const b200dp_md_params& p = *params;
  if (!(p.dt > 0) || (p.ensemble != B200DP_MD_NVE && p.ensemble != B200DP_MD_NVT && p.ensemble != B200DP_MD_NPT))
    return B200DP_ERR_INVALID;
  if (p.ensemble != B200DP_MD_NVE && (p.chain < 1 || p.chain > kMaxChain || !(p.t_target > 0) || !(p.t_damp > 0)))
    return B200DP_ERR_INVALID;
  if (p.ensemble == B200DP_MD_NPT &&
      (p.pchain < 1 || p.pchain > kMaxChain || !(p.p_damp > 0) || box[1] != 0 || box[2] != 0 || box[3] != 0 ||
       box[5] != 0 || box[6] != 0 || box[7] != 0))
    return B200DP_ERR_INVALID;  // isotropic barostat on an orthorhombic box
  if (!vel && !(p.t_init > 0)) return B200DP_ERR_INVALID;
  if (p.rebuild_every < 0 || (p.rebuild_every > 1 && !(p.skin > 0))) return B200DP_ERR_INVALID;
  b200dp_model_info info;
  if (b200dp_model_info_get(engine, &info) != B200DP_OK) return B200DP_ERR_INVALID;
  std::vector<double> mass(natoms), minv(natoms);
  for (int i = 0; i < natoms; ++i) {
    if (atype[i] < 0 || atype[i] >= info.ntypes || atype[i] >= 8 || !(p.mass[atype[i]] > 0)) return B200DP_ERR_BAD_TYPE;
    mass[i] = p.mass[atype[i]];
    minv[i] = 1.0 / mass[i];
  }
  auto* md = new b200dp_md();
  md->engine = engine;
  // skin candidates rebuilt at least every rebuild_every steps and on any step where an atom moved more
  // than skin / 2 (decided on the device); 0 or 1: every step from scratch
  if (b200dp_set_neighbor_reuse(engine, p.skin, p.rebuild_every > 1 ? p.rebuild_every : 0) != B200DP_OK) {
    delete md;
    return B200DP_ERR_INVALID;
  }
  md->p = p;
  md->n = natoms;
  md->ensemble = p.ensemble;
  std::memcpy(md->box, box, sizeof(md->box));
  md->volume = std::fabs(box[0] * (box[4] * box[8] - box[5] * box[7]) - box[1] * (box[3] * box[8] - box[5] * box[6]) +
                         box[2] * (box[3] * box[7] - box[4] * box[6]));
  md->dof = 3.0 * natoms - 3.0;  // centre-of-mass motion removed, as LAMMPS' default temperature compute
  // velocities: given, or seeded Gaussian at t_init with zero total momentum, scaled to t_init exactly
  std::vector<double> v(3 * (size_t)natoms);
  if (vel) {
    std::copy(vel, vel + 3 * (size_t)natoms, v.begin());
  } else {
    init_velocities(natoms, mass.data(), p.t_init, p.seed, md->dof, v.data());
  }
  double mv2 = 0;
  for (int i = 0; i < natoms; ++i)
    for (int c = 0; c < 3; ++c) mv2 += mass[i] * v[3 * i + c] * v[3 * i + c];
  // chain parameters and state
  ChainParams& cp = md->cp;
  Chain ch;
  std::memset(&ch, 0, sizeof(ch));
  ch.factor = 1.0;
  ch.t_current = mv2 * kMvv2e / (md->dof * kBoltz);
  if (p.ensemble != B200DP_MD_NVE) {
    const double w = 1.0 / p.t_damp;
    cp.M = p.chain;
    cp.dof_boltz = md->dof * kBoltz;
    cp.ke_target = md->dof * kBoltz * p.t_target;
    cp.boltz_t = kBoltz * p.t_target;
    cp.dt4 = 0.25 * p.dt;
    cp.dt8 = 0.125 * p.dt;
    cp.dthalf = 0.5 * p.dt;
    cp.mass[0] = cp.ke_target / (w * w);
    for (int i = 1; i < cp.M; ++i) cp.mass[i] = cp.boltz_t / (w * w);
    for (int i = 1; i < cp.M; ++i)
      ch.eta_dotdot[i] = (cp.mass[i - 1] * ch.eta_dot[i - 1] * ch.eta_dot[i - 1] - cp.boltz_t) / cp.mass[i];
  }
  const size_t n3 = 3 * (size_t)natoms;
  cudaError_t ce = cudaSuccess;
  auto chk = [&](cudaError_t e) {
    if (ce == cudaSuccess) ce = e;
  };
  chk(cudaStreamCreateWithFlags(&md->stream, cudaStreamNonBlocking));
  chk(md->x.alloc(n3));
  chk(md->v.alloc(n3));
  chk(md->f.alloc(n3));
  chk(md->minv.alloc(natoms));
  chk(md->mass.alloc(natoms));
  chk(md->e.alloc(1));
  chk(md->vir.alloc(9));
  chk(md->part.alloc(kRedBlocks));
  chk(md->ke.alloc(1));
  chk(md->atype.alloc(natoms));
  chk(md->chain.alloc(1));
  if (ce == cudaSuccess) {
    chk(cudaMemcpy(md->x.p, coord, sizeof(double) * n3, cudaMemcpyHostToDevice));
    chk(cudaMemcpy(md->v.p, v.data(), sizeof(double) * n3, cudaMemcpyHostToDevice));
    chk(cudaMemcpy(md->minv.p, minv.data(), sizeof(double) * natoms, cudaMemcpyHostToDevice));
    chk(cudaMemcpy(md->mass.p, mass.data(), sizeof(double) * natoms, cudaMemcpyHostToDevice));
    chk(cudaMemcpy(md->atype.p, atype, sizeof(int) * natoms, cudaMemcpyHostToDevice));
    chk(cudaMemcpy(md->chain.p, &ch, sizeof(ch), cudaMemcpyHostToDevice));
  }
  if (ce != cudaSuccess) {
    if (md->stream) cudaStreamDestroy(md->stream);
    delete md;
    return B200DP_ERR_CUDA;
  }
  if (p.ensemble == B200DP_MD_NPT) {
    const double w = 1.0 / p.t_damp, wp = 1.0 / p.p_damp, kt = kBoltz * p.t_target;
    md->tch.init(p.chain, cp.mass[0], p.chain > 1 ? cp.mass[1] : 0.0, cp.boltz_t);
    md->pch.init(p.pchain, kt / (wp * wp), kt / (wp * wp), kt);
    md->w_mass = (natoms + 1) * kt / (wp * wp);
    md->vol0 = md->volume;
    md->t_current = ch.t_current;
    (void)w;
  }
  // forces of the initial configuration
  const b200dp_status rc = b200dp_compute_device(engine, md->stream, natoms, 0, md->x.p, md->atype.p, md->box, nullptr,
                                                 md->e.p, md->f.p, md->vir.p, nullptr, nullptr);
  if (rc != B200DP_OK) {
    cudaStreamDestroy(md->stream);
    delete md;
    return rc;
  }
  count_launch();
  k_md_ke<<<kRedBlocks, kMdThreads, 0, md->stream>>>(natoms, md->v.p, md->mass.p, md->part.p);
  if (p.ensemble == B200DP_MD_NPT) {
    // the device NPT state, with the virial of the initial forces
    double vir[9];
    NptState h;
    std::memset(&h, 0, sizeof(h));
    if (md->npt.alloc(1) != cudaSuccess ||
        cudaMemcpyAsync(vir, md->vir.p, sizeof(vir), cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
        cudaStreamSynchronize(md->stream) != cudaSuccess) {
      cudaStreamDestroy(md->stream);
      delete md;
      return B200DP_ERR_CUDA;
    }
    md->vir_trace = vir[0] + vir[4] + vir[8];
    h.tch = md->tch;
    h.pch = md->pch;
    h.w_mass = md->w_mass;
    h.vol0 = md->vol0;
    h.t_current = md->t_current;
    h.vir_trace = md->vir_trace;
    std::memcpy(h.box, md->box, sizeof(h.box));
    std::memcpy(md->box_ref, md->box, sizeof(md->box_ref));
    if (cudaMemcpy(md->npt.p, &h, sizeof(h), cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaStreamDestroy(md->stream);
      delete md;
      return B200DP_ERR_CUDA;
    }
  }
  *out = md;
  return cudaGetLastError() == cudaSuccess ? B200DP_OK : B200DP_ERR_CUDA;
}

// One NPT step, LAMMPS fix npt iso order, entirely on the device: the chains,
// the barostat and the box advance in one-thread kernels and the force call
// reads the box from device memory.
static b200dp_status npt_step(b200dp_md* md) {
  const int n = md->n;
  const double dt = md->p.dt, dtf = 0.5 * dt * kFtm2v;
  const int grid = std::min(kRedBlocks * 4, (n + kMdThreads - 1) / kMdThreads);
  const NptParams q = npt_params(md);
  cudaStream_t st = md->stream;
  count_launch();
  k_npt_pre<<<1, 1, 0, st>>>(q, md->npt.p);
  count_launch();
  k_npt_first_dev<<<grid, kMdThreads, 0, st>>>(n, md->x.p, md->v.p, md->f.p, md->minv.p, md->npt.p, dtf, dt);
  const b200dp_status rc = b200dp_compute_device_dbox(md->engine, st, n, md->x.p, md->atype.p, md->box_ref,
                                                      kGridMinScale, npt_box(md), md->e.p, md->f.p, md->vir.p);
  if (rc != B200DP_OK) return rc;
  count_launch();
  k_npt_second_dev<<<kRedBlocks, kMdThreads, 0, st>>>(n, md->v.p, md->f.p, md->minv.p, md->mass.p, dtf, md->npt.p,
                                                      md->part.p);
  count_launch();
  k_npt_post<<<1, 32, 0, st>>>(q, md->npt.p, md->part.p, kRedBlocks, md->vir.p, md->e.p);
  count_launch();
  k_npt_scale<<<grid, kMdThreads, 0, st>>>(n, md->v.p, md->npt.p);
  count_launch();
  k_md_ke<<<kRedBlocks, kMdThreads, 0, st>>>(n, md->v.p, md->mass.p, md->part.p);
  return cudaGetLastError() == cudaSuccess ? B200DP_OK : B200DP_ERR_CUDA;
}

// One step enqueued on the MD stream.
static b200dp_status md_step(b200dp_md* md) {
  if (md->ensemble == B200DP_MD_NPT) return npt_step(md);
  const int n = md->n;
  const double dtf = 0.5 * md->p.dt * kFtm2v, dt = md->p.dt;
  const int grid = std::min(kRedBlocks * 4, (n + kMdThreads - 1) / kMdThreads);
  const bool nvt = md->ensemble == B200DP_MD_NVT;
  cudaStream_t st = md->stream;
  if (nvt) {
    count_launch();
    k_md_chain<<<1, 32, 0, st>>>(md->cp, md->chain.p, nullptr, 0, nullptr);
  }
  count_launch();
  k_md_first<<<grid, kMdThreads, 0, st>>>(n, md->x.p, md->v.p, md->f.p, md->minv.p, nvt ? md->chain.p : nullptr,
                                          dtf, dt);
  const b200dp_status rc = b200dp_compute_device(md->engine, st, n, 0, md->x.p, md->atype.p, md->box, nullptr,
                                                 md->e.p, md->f.p, md->vir.p, nullptr, nullptr);
  if (rc != B200DP_OK) return rc;
  count_launch();
  k_md_second<<<kRedBlocks, kMdThreads, 0, st>>>(n, md->v.p, md->f.p, md->minv.p, md->mass.p, dtf, md->part.p);
  if (nvt) {
    count_launch();
    k_md_chain<<<1, 32, 0, st>>>(md->cp, md->chain.p, md->part.p, kRedBlocks, nullptr);
    count_launch();
    k_md_scale<<<grid, kMdThreads, 0, st>>>(n, md->v.p, md->chain.p);
    count_launch();
    k_md_ke<<<kRedBlocks, kMdThreads, 0, st>>>(n, md->v.p, md->mass.p, md->part.p);
  }
  return B200DP_OK;
}

// Records `len` steps into a graph (the recording executes nothing; the
// caller replays it).  The cycle starts with the scheduled candidate build,
// so every replay repeats the same rebuild cadence.  A failed recording
// leaves the stream usable and the run continues step by step.
static b200dp_status record_cycle(b200dp_md* md, int len) {
  cudaStream_t st = md->stream;
  const int every = md->p.rebuild_every > 1 ? md->p.rebuild_every : 0;
  if (b200dp_set_neighbor_reuse(md->engine, md->p.skin, every) != B200DP_OK) return B200DP_ERR_INVALID;
  if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
    cudaGetLastError();
    md->cycle_failed = true;
    return B200DP_OK;
  }
  b200dp_status rc = B200DP_OK;
  for (int k = 0; k < len && rc == B200DP_OK; ++k) rc = md_step(md);
  cudaGraph_t g = nullptr;
  const cudaError_t ce = cudaStreamEndCapture(st, &g);
  cudaGraphExec_t ex = nullptr;
  if (rc == B200DP_OK && ce == cudaSuccess && g && cudaGraphInstantiate(&ex, g, 0) == cudaSuccess) {
    md->cycle = ex;
    md->cycle_len = len;
  } else {
    md->cycle_failed = true;
    cudaGetLastError();
  }
  if (g) cudaGraphDestroy(g);
  if (rc != B200DP_OK) return rc;
  // the engine's host-side neighbour cycle advanced during the recording as the
  // replays will advance the device state (a cycle ends where the next one's
  // scheduled build begins); after a failed recording nothing ran: restart it
  if (!md->cycle) return b200dp_set_neighbor_reuse(md->engine, md->p.skin, every);
  return B200DP_OK;
}

b200dp_status b200dp_md_run(b200dp_md* md, int nsteps) {
  if (!md || nsteps < 0) return B200DP_ERR_INVALID;
  for (int s = 0; s < nsteps;) {
    // whole cycles replay the recorded graph; the rest (and a first cycle that
    // is being recorded) are enqueued step by step
    const int L = md->p.rebuild_every > 1 ? md->p.rebuild_every : 1;
    if (md->cycle && nsteps - s >= md->cycle_len) {
      if (cudaGraphLaunch(md->cycle, md->stream) != cudaSuccess) return B200DP_ERR_CUDA;
      md->step += md->cycle_len;
      s += md->cycle_len;
      continue;
    }
    if (!md->cycle && !md->cycle_failed && nsteps - s >= L) {
      const b200dp_status rc = record_cycle(md, L);
      if (rc != B200DP_OK) return rc;
      if (md->cycle) continue;
    }
    const b200dp_status rc = md_step(md);
    if (rc != B200DP_OK) return rc;
    ++md->step;
    ++s;
  }
  return cudaGetLastError() == cudaSuccess ? B200DP_OK : B200DP_ERR_CUDA;
}

b200dp_status b200dp_md_thermo(b200dp_md* md, double* thermo) {
  if (!md || !thermo) return B200DP_ERR_INVALID;
  double e = 0, vir[9], part[kRedBlocks];
  Chain ch;
  if (cudaMemcpyAsync(&e, md->e.p, sizeof(double), cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
      cudaMemcpyAsync(vir, md->vir.p, sizeof(vir), cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
      cudaMemcpyAsync(part, md->part.p, sizeof(part), cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
      cudaMemcpyAsync(&ch, md->chain.p, sizeof(ch), cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
      cudaStreamSynchronize(md->stream) != cudaSuccess)
    return B200DP_ERR_CUDA;
  b200dp_status rc = b200dp_check(md->engine);
  if (rc != B200DP_OK) return rc;
  if (md->ensemble == B200DP_MD_NPT && (rc = npt_refresh(md)) != B200DP_OK) return rc;
  double mv2 = 0;
  for (int k = 0; k < kRedBlocks; ++k) mv2 += part[k];
  const double ke = 0.5 * mv2 * kMvv2e;
  const double temp = 2.0 * ke / (md->dof * kBoltz);
  double e_chain = 0;
  if (md->ensemble == B200DP_MD_NPT) {
    const double kt = kBoltz * md->p.t_target;
    e_chain = md->tch.energy(md->cp.ke_target, kt) + md->pch.energy(kt, kt) +
              1.5 * md->w_mass * md->omega_dot * md->omega_dot + md->p.p_target * (md->volume - md->vol0) / kNktv2p;
  } else if (md->ensemble == B200DP_MD_NVT) {
    const ChainParams& cp = md->cp;
    e_chain = cp.ke_target * ch.eta[0];
    for (int i = 1; i < cp.M; ++i) e_chain += cp.boltz_t * ch.eta[i];
    for (int i = 0; i < cp.M; ++i) e_chain += 0.5 * cp.mass[i] * ch.eta_dot[i] * ch.eta_dot[i];
  }
  thermo[0] = (double)md->step;
  thermo[1] = e;
  thermo[2] = ke;
  thermo[3] = temp;
  thermo[4] = e + ke + e_chain;
  thermo[5] = (md->dof * kBoltz * temp + vir[0] + vir[4] + vir[8]) / (3.0 * md->volume) * kNktv2p;
  thermo[6] = md->volume;
  thermo[7] = e_chain;
  return B200DP_OK;
}

b200dp_status b200dp_md_state(b200dp_md* md, double* coord, double* vel, double* force) {
  if (!md) return B200DP_ERR_INVALID;
  const size_t b = sizeof(double) * 3 * (size_t)md->n;
  if ((coord && cudaMemcpyAsync(coord, md->x.p, b, cudaMemcpyDeviceToHost, md->stream) != cudaSuccess) ||
      (vel && cudaMemcpyAsync(vel, md->v.p, b, cudaMemcpyDeviceToHost, md->stream) != cudaSuccess) ||
      (force && cudaMemcpyAsync(force, md->f.p, b, cudaMemcpyDeviceToHost, md->stream) != cudaSuccess) ||
      cudaStreamSynchronize(md->stream) != cudaSuccess)
    return B200DP_ERR_CUDA;
  return b200dp_check(md->engine);
}

b200dp_status b200dp_md_snapshot_bytes(const b200dp_md* md, size_t* bytes) {
  if (!md || !bytes) return B200DP_ERR_INVALID;
  *bytes = SnapLayout(md->n).total;
  return B200DP_OK;
}

b200dp_status b200dp_md_snapshot(b200dp_md* md, void* d_buf) {
  if (!md || !d_buf) return B200DP_ERR_INVALID;
  const SnapLayout L(md->n);
  // (NPT: the chains, barostat and box are copied from their device state below;
  // the header's copies are informational)
  SnapHeader& h = md->snap_stage;
  std::memset(&h, 0, sizeof(h));
  std::memcpy(h.magic, kSnapMagic, sizeof(h.magic));
  h.n = md->n;
  h.ensemble = md->ensemble;
  h.step = md->step;
  std::memcpy(h.box, md->box, sizeof(h.box));
  h.volume = md->volume;
  h.dof = md->dof;
  h.tch = md->tch;
  h.pch = md->pch;
  h.cp = md->cp;
  h.omega_dot = md->omega_dot;
  h.w_mass = md->w_mass;
  h.vol0 = md->vol0;
  h.t_current = md->t_current;
  h.vir_trace = md->vir_trace;
  h.epot = md->epot;
  h.dt = md->p.dt;
  h.bytes = L.total;
  auto* b = static_cast<unsigned char*>(d_buf);
  const size_t n3 = sizeof(double) * 3 * (size_t)md->n;
  cudaStream_t st = md->stream;
  const auto d2d = cudaMemcpyDeviceToDevice;
  if (cudaMemcpyAsync(b, &h, sizeof(h), cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.x, md->x.p, n3, d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.v, md->v.p, n3, d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.f, md->f.p, n3, d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.e, md->e.p, sizeof(double), d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.vir, md->vir.p, 9 * sizeof(double), d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.part, md->part.p, kRedBlocks * sizeof(double), d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(b + L.chain, md->chain.p, sizeof(Chain), d2d, st) != cudaSuccess ||
      (md->npt.p && cudaMemcpyAsync(b + L.npt, md->npt.p, sizeof(NptState), d2d, st) != cudaSuccess))
    return B200DP_ERR_CUDA;
  return B200DP_OK;
}

b200dp_status b200dp_md_restore(b200dp_md* md, const void* d_buf) {
  if (!md || !d_buf) return B200DP_ERR_INVALID;
  const SnapLayout L(md->n);
  const auto* b = static_cast<const unsigned char*>(d_buf);
  SnapHeader h;
  cudaStream_t st = md->stream;
  if (cudaMemcpyAsync(&h, b, sizeof(h), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return B200DP_ERR_CUDA;
  if (std::memcmp(h.magic, kSnapMagic, sizeof(h.magic)) != 0 || h.n != md->n || h.ensemble != md->ensemble ||
      h.bytes != L.total || h.dt != md->p.dt)
    return B200DP_ERR_INVALID;  // not a snapshot of this system and integrator
  const size_t n3 = sizeof(double) * 3 * (size_t)md->n;
  const auto d2d = cudaMemcpyDeviceToDevice;
  if (cudaMemcpyAsync(md->x.p, b + L.x, n3, d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(md->v.p, b + L.v, n3, d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(md->f.p, b + L.f, n3, d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(md->e.p, b + L.e, sizeof(double), d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(md->vir.p, b + L.vir, 9 * sizeof(double), d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(md->part.p, b + L.part, kRedBlocks * sizeof(double), d2d, st) != cudaSuccess ||
      cudaMemcpyAsync(md->chain.p, b + L.chain, sizeof(Chain), d2d, st) != cudaSuccess ||
      (md->npt.p && cudaMemcpyAsync(md->npt.p, b + L.npt, sizeof(NptState), d2d, st) != cudaSuccess))
    return B200DP_ERR_CUDA;
  md->step = h.step;
  std::memcpy(md->box, h.box, sizeof(md->box));
  md->volume = h.volume;
  md->dof = h.dof;
  md->tch = h.tch;
  md->pch = h.pch;
  md->cp = h.cp;
  md->omega_dot = h.omega_dot;
  md->w_mass = h.w_mass;
  md->vol0 = h.vol0;
  md->t_current = h.t_current;
  md->vir_trace = h.vir_trace;
  md->epot = h.epot;
  if (md->npt.p) {  // the device state is the restored one; its host copies follow it
    const b200dp_status rc = npt_refresh(md);
    if (rc != B200DP_OK) return rc;
  }
  // candidates are rebuilt from the restored positions on the next step
  return b200dp_set_neighbor_reuse(md->engine, md->p.skin, md->p.rebuild_every > 1 ? md->p.rebuild_every : 0);
}

b200dp_status b200dp_md_write_restart(b200dp_md* md, const char* path) {
  if (!md || !path) return B200DP_ERR_INVALID;
  const SnapLayout L(md->n);
  void* d = nullptr;
  if (cudaMalloc(&d, L.total) != cudaSuccess) return B200DP_ERR_CUDA;
  std::vector<unsigned char> host(L.total);
  b200dp_status rc = b200dp_md_snapshot(md, d);
  if (rc == B200DP_OK && (cudaMemcpyAsync(host.data(), d, L.total, cudaMemcpyDeviceToHost, md->stream) != cudaSuccess ||
                          cudaStreamSynchronize(md->stream) != cudaSuccess))
    rc = B200DP_ERR_CUDA;
  cudaFree(d);
  if (rc != B200DP_OK) return rc;
  FILE* fp = std::fopen(path, "wb");
  if (!fp) return B200DP_ERR_IO;
  const bool ok = std::fwrite(host.data(), 1, host.size(), fp) == host.size();
  if (std::fclose(fp) != 0 || !ok) return B200DP_ERR_IO;
  return b200dp_check(md->engine);
}

b200dp_status b200dp_md_read_restart(b200dp_md* md, const char* path) {
  if (!md || !path) return B200DP_ERR_INVALID;
  const SnapLayout L(md->n);
  std::vector<unsigned char> host(L.total);
  FILE* fp = std::fopen(path, "rb");
  if (!fp) return B200DP_ERR_IO;
  const bool ok = std::fread(host.data(), 1, host.size(), fp) == host.size() && std::fgetc(fp) == EOF;
  std::fclose(fp);
  if (!ok) return B200DP_ERR_IO;
  void* d = nullptr;
  if (cudaMalloc(&d, L.total) != cudaSuccess) return B200DP_ERR_CUDA;
  b200dp_status rc = B200DP_OK;
  if (cudaMemcpyAsync(d, host.data(), L.total, cudaMemcpyHostToDevice, md->stream) != cudaSuccess) rc = B200DP_ERR_CUDA;
  if (rc == B200DP_OK) rc = b200dp_md_restore(md, d);
  if (cudaStreamSynchronize(md->stream) != cudaSuccess && rc == B200DP_OK) rc = B200DP_ERR_CUDA;
  cudaFree(d);
  return rc;
}

b200dp_status b200dp_md_destroy(b200dp_md* md) {
  if (!md) return B200DP_OK;
  cudaStreamSynchronize(md->stream);
  if (md->cycle) cudaGraphExecDestroy(md->cycle);
  cudaStreamDestroy(md->stream);
  b200dp_set_neighbor_reuse(md->engine, 0.0, 0);  // the engine's other callers bin from scratch again
  delete md;
  return B200DP_OK;
}

}  // extern "C"
