// Engine state behind the C ABI (include/b200dp.h).
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <string>
#include <vector>

#include "../../include/b200dp.h"
#include "c8l2.cuh"
#include "embed_tc.cuh"
#include "fit_tc.cuh"
#include "model.hpp"
#include "nlist.cuh"
#include "sea.cuh"

namespace b200dp {

b200dp_status cuda_fail(cudaError_t e, const char* expr, const char* file, int line);

// Grow-only device allocation.  Buffers are only (re)allocated outside the
// hot loop, so a call that fits the current capacity allocates nothing.
struct DevBuf {
  void* ptr = nullptr;
  size_t bytes = 0;
  cudaError_t ensure(size_t need);
  void release();
  template <typename T>
  T* as() const {
    return static_cast<T*>(ptr);
  }
};

struct Engine {
  HostModel hm;
  b200dp_options opt{};
  SeaDev sd{};
  std::string err;
  int maxfit = 1;
  int ch_fwd = 32, ch_bwd = 32;

  // weights
  DevBuf w_emb, w_embT;
  std::vector<std::vector<DevBuf>> fit_w, fit_b;  // [type][layer], last layer = output
  std::vector<double> fit_bo;                     // output bias + bias_atom_e per type

  // neighbour graph
  DevBuf xw, cell_of, cell_count, cell_start, cell_cursor, cell_rec;
  DevBuf nl_j, nl_code, nl_rij, nl_cnt;
  DevBuf acc_f, acc_v, nonfinite;  // fixed-point force / atom-virial accumulators (zero between calls)
  bool acc_fresh = false;
  DevBuf blk_counts, type_start, perm_pos, perm_atom;
  DevBuf cand_start, cand_list, ilist_d;
  // tensor-core embedding path (mixed mode)
  bool use_tc = false;
  bool use_f64t = false;  // fp64 mode: the tiled item kernels (embed_f64.cu) over the compacted edge lists
  DevBuf graph_atype, item_rec;
  DevBuf tc_nets, ecount, eoff, tstart, rec_rt, rec_row, rec_slot, partial, scan_scratch, dTbuf;
  // tensor-core fitting (mixed mode)
  bool use_fit_tc = false;
  FitTcPlan fplan;
  std::vector<FitTcWeights> fitw;
  std::vector<DevBuf> fit_dev;  // owns every pre-tiled weight array
  DevBuf ftile;
  std::array<DevBuf, kFitMaxLayers> At_hi, At_lo, THf, Yf;
  std::array<DevBuf, 2> Z_hi, Z_lo, DYf;
  size_t fit_rows_padded = 0;
  // model activations
  DevBuf Tbuf, Dbuf, dDbuf;
  std::vector<DevBuf> th_l, y_l;
  std::array<DevBuf, 2> dy_l, dz_l;
  DevBuf atom_e, gslot, asm_done, reduce_part, scalars, err_buf;
  // C8L2 profile (the reference's production descriptor)
  bool c8 = false;
  C8Host c8h;
  C8Dev c8m;
  std::vector<DevBuf> c8_dev;  // owns the device copies of the model tensors
  DevBuf c8_state, c8_q;
  std::array<DevBuf, kC8MaxFit> c8_Z, c8_H;
  std::array<DevBuf, 2> c8_dH, c8_dZ;
  // neighbour reuse (skin candidates kept for `vl_every` periodic calls)
  double vl_skin = 0;
  int vl_every = 0, vl_age = 0, vl_n = -1, vl_cap = 0, vl_calls = 0;
  long long vl_sched = 0;  // scheduled candidate builds
  bool vl_valid = false;
  // vl_trig: two per-call displacement flags (ints 0, 1) and the count of
  // displacement-triggered rebuilds (u64 at byte 8)
  DevBuf vl_cj, vl_cc, vl_cnt, vl_xref, vl_ls, vl_stale, vl_trig;
  // peer fold (domain decomposition): this rank's owned-atom accumulator is
  // exported by CUDA IPC; peers add their ghost edges' reverse contributions
  // into it over NVLink
  unsigned char* pf_buf = nullptr;  // [accumulator | flags | positions | rendezvous area] of `pf_cap` owned atoms
  size_t pf_off_nf = 0, pf_off_x = 0, pf_off_sync = 0;
  DevBuf pf_seq, pf_sync_err;  // this rank's rendezvous counter; rendezvous timeouts (sticky until b200dp_check)
  int pf_cap = 0, pf_nranks = 0, pf_rank = 0, pf_nghost = 0;
  bool pf_active = false, pf_has_shift = false;
  std::vector<void*> pf_opened;
  DevBuf pf_ptrs, pf_origin, pf_shift;
  PeerSet peer_set() const {
    return PeerSet{pf_ptrs.as<unsigned char*>(), 0, pf_off_nf, pf_off_x};
  }
  PeerSync peer_sync() const {
    return PeerSync{pf_ptrs.as<unsigned char*>(), pf_off_sync,
                    pf_off_sync + sizeof(unsigned long long) * kPeerMaxRanks, pf_nranks, pf_rank};
  }
  // host-call staging
  DevBuf dt_part, dt_cnt;  // split final fitting backward (few row tiles)
  DevBuf h_coord, h_atype, h_force, h_aviral, h_ae;
  // pinned host block for the host call's scalars and error flags (one D2H, one sync)
  unsigned char* pin = nullptr;
  b200dp_status check_flags(const int* h, int stale);
  // A periodic host call whose shape, host buffers, box and device buffers
  // repeat is recorded once (at its second occurrence) and then replayed as
  // one CUDA graph: copies in, the evaluation, copies out.
  struct HostCallKey {
    int nloc = -1;
    const void* ptrs[5] = {};
    double box[9] = {};
    long long epoch = -1;
    bool operator==(const HostCallKey& o) const;
  };
  HostCallKey hc_key;
  cudaGraphExec_t hc_exec = nullptr;
  long long hc_launches = 0;
  bool hc_failed = false;
  void hc_drop();

  cudaStream_t own_stream = nullptr;
  cudaStream_t last_stream = nullptr;
  bool last_stream_set = false;
  int last_nloc = 0, last_nall = 0;
  long long last_overflow = 0;
  bool timing = false;
  std::array<cudaEvent_t, 6> events{};

  b200dp_status init(const char* path, const b200dp_options* o);
  b200dp_status init_c8(const char* path);
  b200dp_status init_tail();
  template <typename P>
  C8Work<P> c8_work() const;
  template <typename P>
  b200dp_status run_c8(cudaStream_t st, int nloc, int nall, const int* d_atype, double* d_force,
                       double* d_atom_energy, double* d_atom_virial, double* d_energy, double* d_virial);
  void release();
  b200dp_status ensure_buffers(int nloc, int nall, int ncells, int ncand);
  b200dp_status make_grid(int nall, const double* box, const double* region, bool periodic, GridSpec& g);
  FormatSpec format_spec(int nloc, int nall) const;
  TcLists tc_lists(int nloc) const;
  void mark(cudaStream_t st, int k);
  bool last_stream_valid() const { return true; }

  template <typename P>
  b200dp_status run_model(cudaStream_t st, int nloc, int nall, const int* d_atype, double* d_force,
                          double* d_atom_energy, double* d_atom_virial, double* d_energy, double* d_virial);
  b200dp_status finish_assembly(cudaStream_t st, int nloc, int nall, double* d_force, double* d_atom_energy,
                                double* d_atom_virial, double* d_energy, double* d_virial, bool env);
  b200dp_status compute_device(cudaStream_t st, int nloc, int nghost, const double* d_coord, const int* d_atype,
                               const double* box, const double* region, double* d_energy, double* d_force,
                               double* d_virial, double* d_atom_energy, double* d_atom_virial);
  // periodic call whose box lives in device memory (d_box); box_ref x min_scale sizes the grid
  b200dp_status compute_device_dbox(cudaStream_t st, int nloc, const double* d_coord, const int* d_atype,
                                    const double* box_ref, double min_scale, const double* d_box, double* d_energy,
                                    double* d_force, double* d_virial);
  const double* dbox_dev = nullptr;  // set during compute_device_dbox
  double dbox_min = 1.0;
  DevBuf dbox_bb;                    // [B | Binv] of the device box
  // Canonical destination-major graph (n nodes, all local), device pointers.
  b200dp_status compute_graph(cudaStream_t st, int n, const int64_t* d_atype64, const int64_t* d_row_ptr,
                              const uint32_t* d_source, const float* d_edge_vec, double* d_atom_energy,
                              double* d_force, double* d_atom_virial, const RawGeometry& raw = RawGeometry{});
  DevBuf vir32;  // fp32 global virial of the last graph call
  b200dp_status compute_with_nlist(cudaStream_t st, int nloc, int nall, const double* d_coord, const int* d_atype,
                                   const b200dp_nlist* nl, double* d_energy, double* d_force, double* d_virial,
                                   double* d_atom_energy, double* d_atom_virial);
  b200dp_status compute_host(int nloc, int nghost, const double* coord, const int* atype, const double* box,
                             const b200dp_nlist* nlist, double* energy, double* force, double* virial,
                             double* atom_energy, double* atom_virial);
  b200dp_status check();
  b200dp_status set_neighbor_reuse(double skin, int every);
  b200dp_status neighbor_stats(long long* out);
  b200dp_status fold_export(int cap, void* handle);
  b200dp_status fold_connect(int nranks, int rank, const void* handles);
  b200dp_status fold_origins(int nghost, const int* d_origin, const double* d_shift);
  b200dp_status fold_scale_shifts(cudaStream_t st, const double* ratio);
  b200dp_status halo_publish(cudaStream_t st, int nloc, const double* d_coord);
  b200dp_status halo_gather(cudaStream_t st, int nloc, int nghost, double* d_coord);
  b200dp_status compute_device_fold(cudaStream_t st, int nloc, int nghost, const double* d_coord,
                                    const int* d_atype, const double* region, double* d_energy, double* d_force,
                                    double* d_virial);
  b200dp_status fold_finish(cudaStream_t st, int nloc, double* d_force);
  b200dp_status peer_reduce(cudaStream_t st, int nv, const double* d_in, double* d_out, long long max_polls);
};

}  // namespace b200dp
