// fp64 embedding path (the parity mode) over the compacted edge lists of the
// tensor-core path.  One block per SM takes the work items (kItemRows centre
// rows of one embedding net) whose edges fall in its share of the edge list;
// its kF64Warps warps take the centre rows one at a time and run each row's
// edges in chunks of 8 through the embedding layers as fp64 tensor-core
// products (mma.sync m8n8k4 .f64: the edges are the 8-row M or N extent), the
// net in shared memory once per block and net.  The forward accumulates
// T = R~^T G of the row in chunk order (results do not depend on the schedule);
// the backward recomputes the forward per chunk and forms dG, dR~, dz3, dh2,
// dz2, dh1 and dE/ds, writing per slot the environment-row gradient that the
// assembly chains to r_ij.  Replaces the per-centre SIMT kernels
// (k_descriptor_fwd/bwd) for the [25, 50, 100] embedding; results agree with
// them to fp64 rounding (the sums run in another order).
#pragma once

#include <cuda_runtime.h>

#include "embed_tc.cuh"
#include "sea.cuh"

namespace b200dp {

constexpr int kF64Warps = 12;  // warps per block (one block per SM)

bool f64_tiled_supported(const SeaDev& s);
int embed_f64_grid(const SeaDev& s, bool backward);
// Tq[net][row][4][M1] per net, then T (atom order, / N) and D = T^T T_< (rows in
// the type-grouped order) summed over the nets in a fixed order.
void launch_embed_fwd_f64(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij,
                          const double* emb, double* Tq, double* T, double* D, const int* perm_atom, int nloc);
// dT[row][4][M1] from T and dD (rows), then the backward -> genv (4 doubles per slot).
void launch_embed_bwd_f64(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const double* rij,
                          const double* emb, const double* T, const double* dD, double* dT, double* genv,
                          const int* type_start, const int* perm_atom, int nloc);

}  // namespace b200dp
