// Tensor-core (tcgen05) embedding path of the mixed-precision mode.
//
// Edges are compacted into one list per embedding net (net q = neighbour type,
// or centre type * ntypes + neighbour type for two-sided models), ordered by
// the centre's row in the type-grouped atom order.  A work item is 8
// consecutive centre rows of one net; its edges are processed in subtiles of
// up to 128, two threads per edge (each owns half of every layer's
// features).  Per subtile the embedding layers 2 and 3 run as tcgen05 MMAs
// (bf16 hi/lo split, three products, fp32 accumulation in TMEM) and the
// contraction T^T = G^T R~ runs as a third MMA whose B operand holds each
// edge's environment row in the column block of its centre (8 centres x 4
// components = 32 columns), accumulated in TMEM across the item's subtiles.
// The backward recomputes layers 1-3 the same way, forms dG and dR~ (rank-4
// contractions with dT) on the CUDA cores and runs the layer backprop
// (dz3 W3^T, dz2 W2^T) as MMAs.  Per-net T are summed in a fixed order by
// the combine kernel, so results are run-to-run identical.
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "model.hpp"
#include "sea.cuh"

namespace b200dp {

// Embedding widths that have a tensor-core instantiation (three layers).
bool tc_supported(const SeaDev& s);
// Bytes of one packed net (B operands in UMMA layout + fp32 w1, b1, b2, b3).
size_t tc_net_bytes(const SeaDev& s);
// Packs one embedding net on the host.
void tc_pack_net(const SeaDev& s, const std::vector<HostLayer>& net, std::vector<unsigned char>& out);

constexpr int kItemRows = 8;  // centre rows per work item
constexpr int kItemPad = 2;   // items per net padded to a multiple of this (the forward's groups per CTA)

struct TcLists {
  int nloc, nnets, ntypes, type_one_side;
  const int* eoff;        // [nnets*nloc + 1] exclusive scan of per-(net,row) edge counts
  const int* istart;      // [nnets + 1] first work item of each net
  const int* type_start;  // [ntypes + 1] rows of each centre type
  const float4* rt;       // [E] environment row (s, s x/r, s y/r, s z/r)
  const int* row;         // [E] centre row in type-grouped order
  const int* slot;        // [E] slot in the formatted neighbour list
  const int4* items;      // [2 * item capacity] per work item {net, first row, end row, first edge}, {end edge, -, -, -}
};

// Work items per embedding net are padded to whole rounds of the grouped
// kernels; this bounds the item count for buffer sizing.
int tc_item_capacity(const SeaDev& s, int nloc);
// Fills TcLists::items from istart / type_start / eoff (one thread per item).
void launch_item_records(cudaStream_t st, const SeaDev& s, const TcLists& L, int4* items);

void launch_edge_count(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom,
                       const int* atype, const int* cnt, int* ecount);
void launch_edge_compact(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom,
                         const int* atype, const int* cnt, const double* rij, const int* eoff, float4* rt, int* row,
                         int* slot);
// Grid for the persistent kernels (CTAs per SM times SMs).
int embed_tc_grid(const SeaDev& s, bool backward);
// Forward: Tq[net][row][4][M1] = sum over the net's edges of the row of R~ (x) G.
void launch_embed_fwd_tc(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                         float* Tq, int* err);
// T_i = sum over nets (fixed order) / N -> T, D (row order, fp32) and, when
// Dt_hi != nullptr, D pre-tiled for the tensor-core fitting (padded rows from
// ftile).  T is [atom][4][M1] unless tiled, then [tile][4][M1][128] in the
// fitting's padded row tiles (what the fused final backward and, when the
// descriptor is formed inside the layer-0 GEMM, its producers read).
void launch_t_combine(cudaStream_t st, const SeaDev& s, const TcLists& L, const int* perm_atom, const int* ftile,
                      const float* Tq, float* T, float* D, unsigned char* Dt_hi, unsigned char* Dt_lo, bool tiled);
// dE/dT per centre row (scaled by 1/N) from T (atom order) and dE/dD (row order).
void launch_dT(cudaStream_t st, const SeaDev& s, int nloc, const int* type_start, const int* perm_atom, const float* T,
               const float* dD, float* dT);
// Embedding backward: recomputes the forward per subtile, then dG, dR~ (CUDA
// cores) and the layer backprop (tensor cores) -> genv, per slot the gradient
// of the energy with respect to the environment row R~ = (sw/r, sw x/r^2,
// sw y/r^2, sw z/r^2) (sw the smooth switch of r) in fp64: [4 slot] = dE/dR~_0
// (through both the embedding input and the contraction), [4 slot + 1..3] =
// dE/dR~_1..3.  The
// assembly (launch_assemble with an environment gradient) applies the chain
// rule to r_ij.
void launch_embed_bwd_tc(cudaStream_t st, const SeaDev& s, const TcLists& L, int grid, const unsigned char* nets,
                         const float* dT, double* genv, int* err);
// Device error slot written by the tensor-core kernels when a bounded wait expires.
constexpr int kErrTcTimeout = 3;

}  // namespace b200dp
