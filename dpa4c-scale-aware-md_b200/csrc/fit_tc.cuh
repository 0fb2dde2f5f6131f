// Tensor-core fitting net (mixed mode): per centre type, the MLP
// D -> h1 -> h2 -> ... -> E and its analytic input gradient dE/dD, as a chain
// of tcgen05 GEMMs over 128-row atom tiles with fused epilogues.
//
// Reference role: the fitting forward + input gradient of
// components/deepmd-op/overlays/op/pt/graph_fitting.cu:614-801 (cuBLAS SGEMM
// plus elementwise epilogues there; wmma FP16 hi/lo "K3N" kernels in
// components/deepmd-op/overlays/op/pt/k3n_fitting.cuh).  Here every operand is
// stored in HBM pre-tiled in the UMMA K-major no-swizzle layout (bf16 hi and lo
// halves, 128 x 32 blocks for activations, BN x 32 blocks for weights), so a
// K chunk is one contiguous cp.async.bulk copy per half.
#pragma once

#include <cuda_runtime.h>

#include <functional>
#include <vector>

#include "model.hpp"
#include "sea.cuh"

namespace b200dp {

constexpr int kFitMaxLayers = 5;
constexpr int kFitBK = 32;

struct FitTcPlan {
  int L = 0;                      // hidden layers
  int dim = 0;                    // descriptor width (K of layer 0)
  int width[kFitMaxLayers] = {};  // hidden widths
  int kpad[kFitMaxLayers] = {};   // padded K of each layer's input
  int res[kFitMaxLayers] = {};    // residual on layer l
  int bn_out = 0;                 // N chunk of the final dE/dD GEMM (fused with dE/dT)
  int bnf[kFitMaxLayers] = {};    // N tile of each forward layer (the last one keeps whole rows)
  int bnb[kFitMaxLayers] = {};    // N tile of each backward layer
  bool ok = false;
  bool chain = false;             // layers 1 .. L-1 (forward and backward) in one launch
  int chain_stages = 0;
};

FitTcPlan fit_tc_plan(const HostModel& m);

// Bytes of one pre-tiled operand of R rows (padded to 128) and K columns.
inline size_t tiled_bytes(size_t rows_padded, int kpad) { return rows_padded * (size_t)kpad * 2; }

// Host packing of a weight matrix as a pre-tiled B operand: element (n, k) for
// n < N, k < Kp, blocks of BN rows x 32, hi and lo halves.
void fit_pack_B(int N, int Kp, int BN, const std::function<double(int, int)>& val, std::vector<unsigned char>& hi,
                std::vector<unsigned char>& lo);

struct FitTcWeights {  // device pointers for one centre type
  const unsigned char* fB_hi[kFitMaxLayers];
  const unsigned char* fB_lo[kFitMaxLayers];
  const unsigned char* bB_hi[kFitMaxLayers];
  const unsigned char* bB_lo[kFitMaxLayers];
  const float* bias[kFitMaxLayers];
  const float* wo;
  double bo;  // output bias + atom energy bias
};

struct FitTcBuffers {
  size_t rows_padded;
  unsigned char* At_hi[kFitMaxLayers];  // tiled input of each forward layer
  unsigned char* At_lo[kFitMaxLayers];
  float* TH[kFitMaxLayers];             // tanh outputs, rows_padded x width (per 128-row tile, column-major)
  float* Y[kFitMaxLayers];              // layer outputs
  unsigned char* Z_hi[2];               // tiled dz ping-pong
  unsigned char* Z_lo[2];
  float* DY[2];                         // residual gradients ping-pong
  // final backward split over several CTAs per row tile (few row tiles):
  // partial second terms [kDtSplitSlots][128][4][16] and per-tile arrival
  // counters [kDtSplitSlots] (zero between launches)
  float* dt_part;
  unsigned* dt_cnt;
};
constexpr int kDtSplitSlots = 148;  // split CTAs of one launch: row tiles x splits <= this

// Whole fitting forward + backward; energies to atom_energy (atom order) and
// dE/dT (rows in type-grouped order, [row][4][M1], through D = T^T T_< with T
// already divided by N and laid out in the fitting's 128-row tiles,
// [tile][4][M1][128], as launch_t_combine writes it) to dT; dE/dD to dD only
// when dD is not null.
void launch_fit_tc(cudaStream_t st, const FitTcPlan& p, int ntypes, int nloc, const int* type_start,
                   const int* ftile, const int* perm_atom, const FitTcWeights* w, const FitTcBuffers& b,
                   double* atom_energy, const float* T, float inv_nnei, float* dT, float* dD, int* err);

}  // namespace b200dp
