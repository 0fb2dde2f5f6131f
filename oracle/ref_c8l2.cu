// Harness around the reference's own C8L2 descriptor kernels (test
// infrastructure only: it generates golden fixtures, see
// tests/golden/make_c8l2_golden.py; nothing on the product path links it).
//
// Compiled by oracle/Makefile (target `ref`) against the reference headers
// where they lie -- include/dpa_chain/graph_compress{,_launch}.{cuh,h} and
// components/deepmd-op/overlays/op/pt/dpa4c/graph_compress_kernel.cuh of the
// dpa4c-runtime project -- into oracle/_ref/libref_c8l2.so.  Only the
// production specialization is instantiated: 8 channels, lmax 2, no radial
// modes, no spin, canonical destination-major rows, uint32 sources
// (the direct engine's configuration, graph_compress.cu:1601-1603).
//
// One call runs the reference forward (descriptor + saved state), then its
// backward (node readout VJP + edge recomputation) for a caller-supplied
// dE/d(descriptor), with every buffer on the device and copied back.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <vector>

#include "graph_compress_kernel.cuh"

namespace {

template <typename T>
T* upload(const T* h, size_t n, cudaError_t& e) {
  T* d = nullptr;
  if (e != cudaSuccess) return nullptr;
  e = cudaMalloc(&d, sizeof(T) * (n ? n : 1));
  if (e == cudaSuccess && n) e = cudaMemcpy(d, h, sizeof(T) * n, cudaMemcpyHostToDevice);
  return d;
}

template <typename T>
T* alloc(size_t n, cudaError_t& e) {
  T* d = nullptr;
  if (e != cudaSuccess) return nullptr;
  e = cudaMalloc(&d, sizeof(T) * (n ? n : 1));
  if (e == cudaSuccess) e = cudaMemset(d, 0, sizeof(T) * (n ? n : 1));
  return d;
}

}  // namespace

extern "C" int ref_c8l2_run(long node_count, long edge_count, const long* row_ptr, const uint32_t* source,
                            const float* edge_vec, const long* atype, int type_count, int interval_count,
                            float table_stride, float table_max, float rcut, float eps, float degree_floor,
                            const float* table, const float* pair_film, const float* type_embedding,
                            const float* readout, const float* output_mean, const float* output_inv_std,
                            const float* descriptor_gradient, float* descriptor, float* state,
                            float* moment_gradient, float* edge_gradient) {
  using namespace deepmd_dpa4c;
  using P = Profile<8, 2, false>;
  if (node_count <= 0 || edge_count < 0) return 1;
  if (row_ptr[0] != 0 || row_ptr[node_count] != edge_count) return 2;
  for (long e = 0; e < edge_count; ++e)
    if (source[e] >= (uint32_t)node_count) return 3;
  for (long n = 0; n < node_count; ++n)
    if (atype[n] < 0 || atype[n] >= type_count) return 4;
  cudaError_t err = cudaSuccess;
  long* d_row = upload(row_ptr, node_count + 1, err);
  uint32_t* d_src = upload(source, edge_count, err);
  float* d_vec = upload(edge_vec, 3 * edge_count, err);
  long* d_type = upload(atype, node_count, err);
  float* d_table = upload(table, (size_t)interval_count * 6 * 8, err);
  float* d_film = upload(pair_film, (size_t)type_count * type_count * 8 * 2, err);
  float* d_temb = upload(type_embedding, (size_t)type_count * 8, err);
  float* d_ro = upload(readout, 8 * 16, err);
  float* d_mean = upload(output_mean, P::OutputWidth, err);
  float* d_istd = upload(output_inv_std, P::OutputWidth, err);
  float* d_dd = upload(descriptor_gradient, (size_t)node_count * P::OutputWidth, err);
  float* d_desc = alloc<float>((size_t)node_count * P::OutputWidth, err);
  float* d_state = alloc<float>((size_t)node_count * P::StateWidth, err);
  float* d_q = alloc<float>((size_t)node_count * P::StateWidth, err);
  float* d_g = alloc<float>((size_t)3 * edge_count, err);
  int rc = err == cudaSuccess ? 0 : 5;
  if (rc == 0) {
    Arguments a{};
    a.node_count = node_count;
    a.edge_count = edge_count;
    a.lmax = 2;
    a.interval_count = interval_count;
    a.type_count = type_count;
    a.table_width = 8;
    a.radial_modes = 0;
    a.node_begin = 0;
    a.clear_padding = false;
    a.coupling_count = 0;
    a.table_stride = table_stride;
    a.table_max = table_max;
    a.rcut = rcut;
    a.eps = eps;
    a.degree_floor = degree_floor;
    a.canonical = true;
    a.has_spin = false;
    a.index_kind = IndexKind::Bits32;
    a.edge_index = d_src;
    a.edge_vec = d_vec;
    a.destination_row_ptr = d_row;
    a.atype = d_type;
    a.table = d_table;
    a.pair_film = d_film;
    a.type_embedding = d_temb;
    a.readout_matrices = d_ro;
    a.output_mean = d_mean;
    a.output_inv_std = d_istd;
    a.descriptor = d_desc;
    a.state_out = d_state;
    ForwardLauncher<8, 2, false, false, true, uint32_t>::run(a, 0);
    a.descriptor_gradient = d_dd;
    a.state = d_state;
    a.moment_gradient = d_q;
    a.edge_gradient = d_g;
    BackwardLauncher<8, 2, false, false, true, uint32_t>::run(a, 0);
    err = cudaDeviceSynchronize();
    if (err == cudaSuccess) err = cudaGetLastError();
    if (err == cudaSuccess)
      err = cudaMemcpy(descriptor, d_desc, sizeof(float) * node_count * P::OutputWidth, cudaMemcpyDeviceToHost);
    if (err == cudaSuccess)
      err = cudaMemcpy(state, d_state, sizeof(float) * node_count * P::StateWidth, cudaMemcpyDeviceToHost);
    if (err == cudaSuccess)
      err = cudaMemcpy(moment_gradient, d_q, sizeof(float) * node_count * P::StateWidth, cudaMemcpyDeviceToHost);
    if (err == cudaSuccess && edge_count)
      err = cudaMemcpy(edge_gradient, d_g, sizeof(float) * 3 * edge_count, cudaMemcpyDeviceToHost);
    if (err != cudaSuccess) {
      std::fprintf(stderr, "ref_c8l2: %s\n", cudaGetErrorString(err));
      rc = 6;
    }
  }
  for (void* p : {(void*)d_row, (void*)d_src, (void*)d_vec, (void*)d_type, (void*)d_table, (void*)d_film,
                  (void*)d_temb, (void*)d_ro, (void*)d_mean, (void*)d_istd, (void*)d_dd, (void*)d_desc,
                  (void*)d_state, (void*)d_q, (void*)d_g})
    if (p) cudaFree(p);
  return rc;
}
