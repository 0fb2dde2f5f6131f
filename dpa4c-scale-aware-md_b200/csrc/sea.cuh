// DPA4C-style (se_e2_a type) model kernels: environment matrix with smooth
// switch, embedding net fused with the contraction T = R~^T G / N and
// D = T^T T_<, the fitting MLP forward and analytic backward, and the
// atomic-free force / virial assembly.
//
// Reference roles these kernels take over (paths in the reference project):
//  - descriptor forward: components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh:78-767
//  - fitting forward + input gradient: components/deepmd-op/overlays/op/pt/graph_fitting.cu:614-801
//  - node/edge backward: graph_compress_kernel.cuh:909-1458, 1460-1917
//  - force / virial assembly: components/deepmd-op/overlays/op/pt/edge_force_virial.cu:1-190
//  - widen + reduce: components/deepmd-op/overlays/op/pt/dpa4c/graph_compress.cu:1493-1504
// The se_e2_a math itself (switch, residual rules, 1/N normalisation) is
// DeePMD-kit's published definition; DeePMD-kit is not vendored in the
// reference (production/dpa4c-runtime/third_party/sources.lock.json:4-12).
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace b200dp {

struct SeaDev {
  int ntypes, nnets, type_one_side, nl;  // nl: embedding layers
  int ed[kMaxLayers + 1];                // embedding dims, ed[0] = 1
  int M1, M2, dim, selt, maxd;
  int sel[kMaxTypes], off[kMaxTypes + 1];
  double rcut, rcut_smth, inv_nnei;
  int net_stride;  // elements per embedding net
  int w_off[kMaxLayers], b_off[kMaxLayers];
};

constexpr int kSeaThreads = 128;

template <typename P>
size_t descriptor_fwd_smem(const SeaDev& s, int ch);
template <typename P>
size_t descriptor_bwd_smem(const SeaDev& s, int ch);

template <typename P>
void launch_descriptor_fwd(cudaStream_t st, const SeaDev& s, int nloc, int ch, int grid, const double* rij,
                           const int* cnt, const int* atype, const int* perm_pos, const P* emb, P* T, P* D);
template <typename P>
void launch_descriptor_bwd(cudaStream_t st, const SeaDev& s, int nloc, int ch, int grid, const double* rij,
                           const int* cnt, const int* atype, const int* perm_pos, const P* emb, const P* embT,
                           const P* T, const P* dD, double* gslot);
template <typename P>
int descriptor_grid(const SeaDev& s, int ch, bool bwd, int nloc);

// Fitting pieces.  Rows of one centre type are [range[0], range[1]) of the
// type-grouped order; `range` is device memory so no host sync is needed.
// Mmax bounds the row count for the launch grid (blocks past range exit).
template <typename P>
void launch_fit_forward_layer(cudaStream_t st, int Mmax, const int* range, int N, int K, const P* X, int ldx,
                              const P* W, const P* b, bool residual, P* th, P* Y);
template <typename P>
void launch_fit_energy(cudaStream_t st, int Mmax, const int* range, int N, const P* Y, const P* wo,
                       double bo_plus_bias, const int* perm_atom, double* atom_energy);
template <typename P>
void launch_fit_seed(cudaStream_t st, int Mmax, const int* range, int N, const P* wo, const P* th, P* dy, P* dz);
// dX = dZ W^T (+ dY_next if residual); if th_prev: dz_prev = dX * (1 - th_prev^2).
template <typename P>
void launch_fit_backward_layer(cudaStream_t st, int Mmax, const int* range, int Nin, int Nout, const P* dZ,
                               const P* W, const P* dY_next, P* dX, const P* th_prev, P* dZ_prev);

// Forces, optional per-atom virials, and the total energy and virial
// (deterministic).  partial holds 10 doubles per assembly block
// (assemble_blocks(nloc)); acc_f (6 x u64 per atom), acc_v (18 x u64 per atom,
// only with atom_virial), nonfinite (one per atom) and *done must be zero
// before the first launch and are zero again after each.
// With env.on, gslot holds per slot the gradient with respect to the
// environment row R~ = (sw/r, sw x/r^2, sw y/r^2, sw z/r^2) (4 doubles; the
// tensor-core backward writes it) and the assembly applies the chain rule to
// r_ij with the cutoffs in env; otherwise dE/dr_ij (3 doubles).
struct EnvChain {
  bool on;
  double rcut, rcut_smth;
};
constexpr int kAssembleMaxSlots = 512;  // neighbour slots per centre (sum of sel) the assembly takes
void launch_assemble(cudaStream_t st, int nloc, int nall, int selt, const int* nl_j, const double* gslot,
                     const double* rij, const double* atom_e, double* force, double* atom_virial,
                     unsigned long long* acc_f, unsigned long long* acc_v, unsigned* nonfinite, double* partial,
                     unsigned* done, double* energy, double* virial, const EnvChain& env);
int assemble_blocks(int nloc);
// Domain decomposition over NVLink peers.  Every rank exports one device
// buffer (CUDA IPC) holding its owned atoms' fixed-point force accumulator
// ([cap][3][lo, hi] u64 at off_acc), their non-finite flags (u32 at off_nf)
// and their published positions ([cap][3] f64 at off_x); base[r] is rank r's
// buffer as mapped in this process.
struct PeerSet {
  unsigned char* const* base;
  size_t off_acc, off_nf, off_x;
};
// Device-side rendezvous of the ranks through their exported buffers: a
// sync area per buffer holds one arrival counter per source rank (u64, at
// off_flags) and two mailboxes of kPeerMaxValues doubles per source rank
// (at off_mail, alternating between consecutive rendezvous).
constexpr int kPeerMaxRanks = 64;
constexpr int kPeerMaxValues = 16;
constexpr size_t kPeerSyncBytes = sizeof(unsigned long long) * kPeerMaxRanks +
                                  sizeof(double) * 2 * kPeerMaxRanks * kPeerMaxValues;
struct PeerSync {
  unsigned char* const* base;  // every rank's buffer as mapped in this process
  size_t off_flags, off_mail;
  int nranks, rank;
};
// One rendezvous of all ranks on `st`: this rank's nv values (device memory,
// nv <= kPeerMaxValues; nv = 0 is a plain barrier) go to every rank's mailbox
// with plain peer stores, then its arrival counter is raised in every rank's
// buffer; the kernel waits until every rank has arrived at this rendezvous
// and writes the sum of all ranks' values, in rank order, to out.  Every rank
// must call it the same number of times in the same order.  The wait is
// bounded: after `limit` polls the kernel adds 1 to err[kErrPeerTimeout],
// writes nothing to out and returns.  `seq` is this rank's device-side
// rendezvous counter (u64, starts at 0).  Ranks must run on different GPUs:
// kernels of one GPU are not guaranteed to run at the same time.
void launch_peer_reduce(cudaStream_t st, const PeerSync& ps, unsigned long long* seq, const double* in, int nv,
                        double* out, int* err, long long limit);
// The assembly with owned neighbours' contributions added to this rank's
// exported accumulator (own_acc, own_nf) and ghost rows (acc_f rows
// nloc..nall) then pushed to their owners' accumulators, origin[g] = (owner
// rank, owner's row) -- no conversion; launch_fold_finish converts this rank's
// accumulator into the owned forces once every rank's push has completed.
void launch_assemble_fold(cudaStream_t st, int nloc, int nall, int selt, const int* nl_j, const double* gslot,
                          const double* rij, const double* atom_e, double* force, unsigned long long* acc_f,
                          unsigned* nonfinite, unsigned long long* own_acc, unsigned* own_nf, const PeerSet& peers,
                          const int2* origin, double* partial, unsigned* done, double* energy, double* virial,
                          const EnvChain& env);
void launch_fold_finish(cudaStream_t st, int nloc, double* force, unsigned long long* acc, unsigned* nonfinite);
// shift [nghost][3] scaled per component by ratio[3] (the box scaled by a barostat).
void launch_scale_shifts(cudaStream_t st, int nghost, double* shift, const double* ratio);
// x rows nloc..nloc+nghost from the owners' published positions (+ shift [nghost][3]).
void launch_halo_gather(cudaStream_t st, int nloc, int nghost, double* x, const PeerSet& peers, const int2* origin,
                        const double* shift);

}  // namespace b200dp
