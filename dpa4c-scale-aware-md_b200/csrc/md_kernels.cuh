// Velocity-Verlet and Nose-Hoover chain kernels shared by the single-GPU MD
// driver (md.cu) and the domain-decomposed one (dd.cu).  Metal units; the
// chain follows LAMMPS FixNH::nhc_temp_integrate (one Suzuki-Yoshida stage),
// as kept on the device by the reference
// (components/lammps/overlays/src/KOKKOS/dpa_fast_step_kokkos.h:307-400).
// Included into an anonymous namespace of each translation unit.
#pragma once

constexpr double kMvv2e = 1.0364269e-4;  // (g/mol) (A/ps)^2 -> eV
constexpr double kFtm2v = 1.0 / 1.0364269e-4;
constexpr double kBoltz = 8.617343e-5;  // eV / K
constexpr double kNktv2p = 1.6021765e6;  // eV / A^3 -> bar
constexpr int kMaxChain = 8;
constexpr int kRedBlocks = 148;
constexpr int kMdThreads = 256;

struct Chain {
  double eta[kMaxChain], eta_dot[kMaxChain + 1], eta_dotdot[kMaxChain];
  double t_current, factor;
};

struct ChainParams {
  int M;
  double dof_boltz, ke_target, boltz_t, dt4, dt8, dthalf;
  double mass[kMaxChain];
};

// v = v * s + dtf F / m ; x += dt v   (s = chain factor, 1 without a thermostat)
__global__ void k_md_first(int n, double* __restrict__ x, double* __restrict__ v, const double* __restrict__ f,
                           const double* __restrict__ minv, const Chain* __restrict__ ch, double dtf, double dt) {
  const double s = ch ? ch->factor : 1.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double w = dtf * minv[i];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double vv = v[3 * i + c] * s + w * f[3 * i + c];
      v[3 * i + c] = vv;
      x[3 * i + c] += dt * vv;
    }
  }
}

// v += dtf F / m, and per-block partial sums of m v^2 (fixed grid, fixed order)
__global__ void __launch_bounds__(kMdThreads) k_md_second(int n, double* __restrict__ v, const double* __restrict__ f,
                                                          const double* __restrict__ minv,
                                                          const double* __restrict__ mass, double dtf,
                                                          double* __restrict__ part) {
  __shared__ double sh[kMdThreads / 32];
  double acc = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const double w = dtf * minv[i];
    double s2 = 0.0;
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const double vv = v[3 * i + c] + w * f[3 * i + c];
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

// sum of the partials in a fixed order (one warp)
__device__ double sum_parts(const double* part, int nparts) {
  const int lane = threadIdx.x & 31;
  double a = 0.0;
  for (int k = lane; k < nparts; k += 32) a += part[k];
  return warp_sum(a);
}

// One half-step of the chain (LAMMPS FixNH::nhc_temp_integrate with one
// Suzuki-Yoshida stage).  With `part` the current temperature comes from the
// kinetic-energy partials, else from the state.  Writes the velocity factor.
__global__ void k_md_chain(ChainParams p, Chain* __restrict__ st, const double* __restrict__ part, int nparts,
                           double* __restrict__ ke_out) {
  double mv2 = 0.0;
  if (part) mv2 = sum_parts(part, nparts);
  if (threadIdx.x != 0) return;
  double t_current = part ? mv2 * kMvv2e / p.dof_boltz : st->t_current;
  if (ke_out && part) *ke_out = 0.5 * mv2 * kMvv2e;
  const int M = p.M;
  double eta_dot[kMaxChain + 1], eta_dotdot[kMaxChain];
  for (int i = 0; i <= M; ++i) eta_dot[i] = st->eta_dot[i];
  for (int i = 0; i < M; ++i) eta_dotdot[i] = st->eta_dotdot[i];
  double ke = p.dof_boltz * t_current;
  eta_dotdot[0] = (ke - p.ke_target) / p.mass[0];
  double expfac = 1.0;
  for (int i = M - 1; i > 0; --i) {
    expfac = exp(-p.dt8 * eta_dot[i + 1]);
    eta_dot[i] = (eta_dot[i] * expfac + eta_dotdot[i] * p.dt4) * expfac;
  }
  expfac = exp(-p.dt8 * eta_dot[1]);
  eta_dot[0] = (eta_dot[0] * expfac + eta_dotdot[0] * p.dt4) * expfac;
  const double factor = exp(-p.dthalf * eta_dot[0]);
  t_current *= factor * factor;
  ke = p.dof_boltz * t_current;
  eta_dotdot[0] = (ke - p.ke_target) / p.mass[0];
  for (int i = 0; i < M; ++i) st->eta[i] += p.dthalf * eta_dot[i];
  eta_dot[0] = (eta_dot[0] * expfac + eta_dotdot[0] * p.dt4) * expfac;
  for (int i = 1; i < M; ++i) {
    expfac = exp(-p.dt8 * eta_dot[i + 1]);
    eta_dotdot[i] = (p.mass[i - 1] * eta_dot[i - 1] * eta_dot[i - 1] - p.boltz_t) / p.mass[i];
    eta_dot[i] = (eta_dot[i] * expfac + eta_dotdot[i] * p.dt4) * expfac;
  }
  for (int i = 0; i <= M; ++i) st->eta_dot[i] = eta_dot[i];
  for (int i = 0; i < M; ++i) st->eta_dotdot[i] = eta_dotdot[i];
  st->t_current = t_current;
  st->factor = factor;
}

__global__ void k_md_scale(int n, double* __restrict__ v, const Chain* __restrict__ ch) {
  const double s = ch->factor;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * n; i += gridDim.x * blockDim.x) v[i] *= s;
}

// kinetic-energy partials only (thermo after creation)
__global__ void __launch_bounds__(kMdThreads) k_md_ke(int n, const double* __restrict__ v,
                                                      const double* __restrict__ mass, double* __restrict__ part) {
  __shared__ double sh[kMdThreads / 32];
  double acc = 0.0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    acc += mass[i] * (v[3 * i] * v[3 * i] + v[3 * i + 1] * v[3 * i + 1] + v[3 * i + 2] * v[3 * i + 2]);
  acc = warp_sum(acc);
  if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double b = 0.0;
    for (int w = 0; w < kMdThreads / 32; ++w) b += sh[w];
    part[blockIdx.x] = b;
  }
}


// splitmix64 + Box-Muller: seeded Gaussian draws for the initial velocities
struct Rng {
  uint64_t s;
  uint64_t next() {
    uint64_t z = (s += 0x9E3779B97F4A7C15ull);
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
  }
  double uniform() { return ((next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }
  double gauss() { return std::sqrt(-2.0 * std::log(uniform())) * std::cos(6.283185307179586 * uniform()); }
};


// Seeded Gaussian velocities at t_init with zero total momentum, scaled so that
// the temperature over `dof` degrees of freedom is t_init exactly (host; the
// same draws for the same seed on every rank of a decomposed run).
inline void init_velocities(int natoms, const double* mass, double t_init, unsigned long long seed, double dof,
                            double* v) {
  Rng rng{seed ? seed : 0x5EEDull};
  double pc[3] = {0, 0, 0}, mt = 0;
  for (int i = 0; i < natoms; ++i) {
    const double sd = std::sqrt(kBoltz * t_init / (mass[i] * kMvv2e));
    for (int c = 0; c < 3; ++c) {
      v[3 * i + c] = sd * rng.gauss();
      pc[c] += mass[i] * v[3 * i + c];
    }
    mt += mass[i];
  }
  double mv2 = 0;
  for (int i = 0; i < natoms; ++i)
    for (int c = 0; c < 3; ++c) {
      v[3 * i + c] -= pc[c] / mt;
      mv2 += mass[i] * v[3 * i + c] * v[3 * i + c];
    }
  const double t_now = mv2 * kMvv2e / (dof * kBoltz);
  const double s = t_now > 0 ? std::sqrt(t_init / t_now) : 0.0;
  for (size_t k = 0; k < 3 * (size_t)natoms; ++k) v[k] *= s;
}

// v = v * sv + dtf F / m ; x = e (e x + dt v)   (NPT first half: remap, drift, remap)
__global__ void k_npt_first(int n, double* __restrict__ x, double* __restrict__ v, const double* __restrict__ f,
                            const double* __restrict__ minv, double sv, double dtf, double dt, double e) {
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

// v = (v + dtf F / m) * sv, with per-block partial sums of m v^2
__global__ void __launch_bounds__(kMdThreads) k_npt_second(int n, double* __restrict__ v,
                                                           const double* __restrict__ f,
                                                           const double* __restrict__ minv,
                                                           const double* __restrict__ mass, double dtf, double sv,
                                                           double* __restrict__ part) {
  __shared__ double sh[kMdThreads / 32];
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

__global__ void k_md_scale_by(int n, double* __restrict__ v, double s) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 3 * n; i += gridDim.x * blockDim.x) v[i] *= s;
}

// Nose-Hoover chain of the NPT path (same recurrence as k_md_chain), usable on
// the host and, as part of the device NPT state, in one-thread kernels.
struct HostChain {
  int M = 0;
  double eta[kMaxChain] = {0}, eta_dot[kMaxChain + 1] = {0}, eta_dotdot[kMaxChain] = {0}, mass[kMaxChain] = {0};
  __host__ __device__ void init(int m, double q0, double qi, double boltz_t) {
    M = m;
    mass[0] = q0;
    for (int i = 1; i < M; ++i) mass[i] = qi;
    for (int i = 1; i < M; ++i) eta_dotdot[i] = (mass[i - 1] * eta_dot[i - 1] * eta_dot[i - 1] - boltz_t) / mass[i];
  }
  // Thermostat half-step for kinetic energy `ke` (target ke_target); returns the velocity factor.
  __host__ __device__ double thermostat(double& t_current, double dof_boltz, double ke_target, double boltz_t, double dt) {
    const double dt4 = 0.25 * dt, dt8 = 0.125 * dt, dthalf = 0.5 * dt;
    eta_dotdot[0] = (dof_boltz * t_current - ke_target) / mass[0];
    double expfac = 1.0;
    for (int i = M - 1; i > 0; --i) {
      expfac = exp(-dt8 * eta_dot[i + 1]);
      eta_dot[i] = (eta_dot[i] * expfac + eta_dotdot[i] * dt4) * expfac;
    }
    expfac = exp(-dt8 * eta_dot[1]);
    eta_dot[0] = (eta_dot[0] * expfac + eta_dotdot[0] * dt4) * expfac;
    const double factor = exp(-dthalf * eta_dot[0]);
    t_current *= factor * factor;
    eta_dotdot[0] = (dof_boltz * t_current - ke_target) / mass[0];
    for (int i = 0; i < M; ++i) eta[i] += dthalf * eta_dot[i];
    eta_dot[0] = (eta_dot[0] * expfac + eta_dotdot[0] * dt4) * expfac;
    for (int i = 1; i < M; ++i) {
      expfac = exp(-dt8 * eta_dot[i + 1]);
      eta_dotdot[i] = (mass[i - 1] * eta_dot[i - 1] * eta_dot[i - 1] - boltz_t) / mass[i];
      eta_dot[i] = (eta_dot[i] * expfac + eta_dotdot[i] * dt4) * expfac;
    }
    return factor;
  }
  // Barostat-chain half-step (FixNH::nhc_press_integrate, isotropic): scales
  // omega_dot; kinetic energy 3 W omega_dot^2 against kB T0.
  __host__ __device__ void barostat(double& omega_dot, double w_mass, double kt, double dt) {
    const double dt4 = 0.25 * dt, dt8 = 0.125 * dt, dthalf = 0.5 * dt;
    double ke = 3.0 * w_mass * omega_dot * omega_dot;
    eta_dotdot[0] = (ke - kt) / mass[0];
    double expfac = 1.0;
    for (int i = M - 1; i > 0; --i) {
      expfac = exp(-dt8 * eta_dot[i + 1]);
      eta_dot[i] = (eta_dot[i] * expfac + eta_dotdot[i] * dt4) * expfac;
    }
    expfac = exp(-dt8 * eta_dot[1]);
    eta_dot[0] = (eta_dot[0] * expfac + eta_dotdot[0] * dt4) * expfac;
    for (int i = 0; i < M; ++i) eta[i] += dthalf * eta_dot[i];
    omega_dot *= exp(-dthalf * eta_dot[0]);
    ke = 3.0 * w_mass * omega_dot * omega_dot;
    eta_dotdot[0] = (ke - kt) / mass[0];
    eta_dot[0] = (eta_dot[0] * expfac + eta_dotdot[0] * dt4) * expfac;
    for (int i = 1; i < M; ++i) {
      expfac = exp(-dt8 * eta_dot[i + 1]);
      eta_dotdot[i] = (mass[i - 1] * eta_dot[i - 1] * eta_dot[i - 1] - kt) / mass[i];
      eta_dot[i] = (eta_dot[i] * expfac + eta_dotdot[i] * dt4) * expfac;
    }
  }
  __host__ __device__ double energy(double first_kt, double kt) const {
    double e = first_kt * eta[0];
    for (int i = 1; i < M; ++i) e += kt * eta[i];
    for (int i = 0; i < M; ++i) e += 0.5 * mass[i] * eta_dot[i] * eta_dot[i];
    return e;
  }
};

