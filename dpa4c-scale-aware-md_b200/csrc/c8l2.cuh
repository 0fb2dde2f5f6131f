// C8L2 profile: the reference's production descriptor ("DPA4C-Nano": 8 scalar
// channels, angular degrees <= 2, tabulated radial branch, PairFiLM amplitude,
// Gram / bispectrum / quartic invariants) with its shared SiLU fitting net,
// node-readout VJP and edge recomputation.  Kernels are templated on the
// arithmetic type P: float reproduces the reference's fp32 path, double is
// the fp64 mode.  The edge list is the formatted neighbour list (kept slots),
// and dE/dr per slot feeds the shared force / virial assembly.
//
// Replaces components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh
// (forward_kernel :78-767, node_backward_kernel :909-1458,
// edge_backward_kernel :1460-1917) and the fitting of
// components/deepmd-op/overlays/op/pt/graph_fitting.cu of the dpa4c-runtime
// project, on the formatted list of this framework.
#pragma once

#include <cuda_runtime.h>

namespace b200dp {

constexpr int kC8Channels = 8;
constexpr int kC8Dim = 70;    // descriptor width
constexpr int kC8State = 42;  // 40 normalized moments + scalar and angular normalizers
constexpr int kC8MaxFit = 4;  // fitting layers

// Device-resident model.  Array pointers hold the arithmetic type P of the
// engine (float or double); bias_atom_e stays fp64.
struct C8Dev {
  int ntypes = 0, nint = 0, nfit = 0, act = 1;
  double stride = 0, rcut = 0, eps = 0, floor_ = 0, b_head = 0;
  const void* table = nullptr;    // [nint][6 * 8]: quartet block [8][c0..c3], pair block [8][c4, c5]
  const void* film = nullptr;     // [ntypes^2][8][2]
  const void* temb = nullptr;     // [ntypes][8]
  const void* readout = nullptr;  // [8][4][4]
  const void* mean = nullptr;     // [70]
  const void* istd = nullptr;     // [70]
  const void* fw[kC8MaxFit] = {};
  const void* fb[kC8MaxFit] = {};
  int fdin[kC8MaxFit] = {}, fdout[kC8MaxFit] = {}, fres[kC8MaxFit] = {};
  const void* w_head = nullptr;
  const double* bias = nullptr;  // bias_atom_e [ntypes]
};

// Per-node buffers of one evaluation (type P): the fitting keeps its
// pre-activations Z[l] and outputs H[l] for the backward; dH and dZ
// alternate between two buffers.
template <typename P>
struct C8Work {
  P* desc;   // [n][70]
  P* state;  // [n][42]
  P* dD;     // [n][70]
  P* q;      // [n][42]
  P* Z[kC8MaxFit];
  P* H[kC8MaxFit];
  P* dH[2];
  P* dZ[2];
};

template <typename P>
void launch_c8_forward(cudaStream_t st, const C8Dev& m, int nloc, int selt, const int* nl_j, const double* rij,
                       const int* atype, const C8Work<P>& w);
template <typename P>
void launch_c8_fitting(cudaStream_t st, const C8Dev& m, int nloc, const int* atype, const C8Work<P>& w,
                       double* atom_e);
template <typename P>
void launch_c8_node_backward(cudaStream_t st, const C8Dev& m, int nloc, const C8Work<P>& w);
template <typename P>
void launch_c8_edge_backward(cudaStream_t st, const C8Dev& m, int nloc, int selt, const int* nl_j,
                             const double* rij, const int* atype, const C8Work<P>& w, double* gslot);

}  // namespace b200dp
