/*
 * b200dp — B200-native DPA4C-style energy / force / virial evaluation.
 *
 * C ABI of the force-evaluation hot path.  Plain pointers and sizes only; no
 * C++ or torch types cross this boundary, and no exception leaves it: every
 * call returns a b200dp_status and the engine keeps a readable message.
 *
 * Interfaces this header replaces (paths inside the reference project):
 *
 *  - DeePMD C++ API, DeepPot::compute(ener, force, virial, atom_energy,
 *    atom_virial, coord, atype, box[, nghost, lmp_list, ago])
 *    components/deepmd-op/overlays/api_cc/include/DeepPot.h:605-690
 *      -> b200dp_compute_host / b200dp_compute_host_nlist
 *  - DeepPot::compute_canonical_graph_gpu (device pointers, caller's stream)
 *    components/deepmd-op/overlays/api_cc/include/DeepPot.h:903-915
 *      -> b200dp_compute_device
 *  - extern "C" dpa_direct_energy_force(atype, row_ptr, source, edge_vec,
 *    node_count, nloc, edge_storage, energy, force, virial)
 *    components/deepmd-op/overlays/op/pt/dpa4c/graph_compress.cu:1817-1902
 *      -> b200dp_direct_energy_force (same argument meaning and return
 *         convention: 1 = handled, 0 = caller must fall back)
 *  - DeepPotPTExpt::init (model load and priming)
 *    components/deepmd-op/overlays/api_cc/src/DeepPotPTExpt.cc:324
 *      -> b200dp_create
 *
 * Units follow DeePMD/LAMMPS metal units: Angstrom, eV, eV/Angstrom.
 * Virial: 9 components, row-major, W[a][b] = sum over edges of -g_a * r_b
 * (g = dE/dr_ij, r_ij = x_j - x_i); the atom virial of an edge belongs to the
 * neighbour j, as in the reference's edge assembly
 * (components/deepmd-op/overlays/op/pt/edge_force_virial.cu:8-11).
 */
#ifndef B200DP_H
#define B200DP_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum b200dp_status {
  B200DP_OK = 0,
  B200DP_ERR_INVALID = 1,      /* bad argument (null pointer, negative size, ...) */
  B200DP_ERR_IO = 2,           /* model file missing or malformed */
  B200DP_ERR_CUDA = 3,         /* a CUDA runtime call failed; see b200dp_last_error */
  B200DP_ERR_SEL_OVERFLOW = 4, /* a type section held more neighbours than sel (only
                                  when b200dp_options.sel_overflow_is_error != 0;
                                  otherwise the nearest sel are kept, as DeePMD does) */
  B200DP_ERR_CAPACITY = 5,     /* a centre had more in-cutoff candidates than the
                                  builder's per-centre buffer */
  B200DP_ERR_BAD_TYPE = 6,     /* an atom type outside [0, ntypes) */
  B200DP_ERR_UNSUPPORTED = 7,  /* configuration this build does not handle */
  B200DP_ERR_PEER_TIMEOUT = 8  /* a device-side rendezvous of the ranks (b200dp_peer_reduce) gave up
                                  waiting: another rank never arrived */
} b200dp_status;

typedef enum b200dp_precision {
  B200DP_FP64 = 0,  /* every stage in fp64 */
  B200DP_MIXED = 1  /* fp64 geometry and accumulation, fp32 networks */
} b200dp_precision;

typedef struct b200dp_options {
  int precision;              /* b200dp_precision */
  int device;                 /* CUDA device ordinal */
  int sel_overflow_is_error;  /* 0: truncate to sel like DeePMD; 1: report B200DP_ERR_SEL_OVERFLOW */
  int simt_only;              /* 1: never use the tensor-core kernels (mixed mode uses SIMT fp32) */
  int keep_descriptor;        /* 1: keep D and dE/dD of the last call for b200dp_last_descriptor (the
                                 tensor-core mixed path otherwise never materialises them) */
  int reserved[11];
} b200dp_options;

typedef struct b200dp_model_info {
  int ntypes;
  int sel_total;
  int descriptor_dim;
  int embedding_out;  /* M1 */
  int axis;           /* M2 */
  int n_embedding_layers;
  int n_fitting_layers;
  int type_one_side;
  double rcut;
  double rcut_smth;
} b200dp_model_info;

/* LAMMPS-style full neighbour list (DeePMD's InputNlist: inum, ilist,
 * numneigh, firstneigh).  Candidates may include skin neighbours; the
 * engine re-applies the cutoff and the per-type sel ordering. */
typedef struct b200dp_nlist {
  int inum;
  const int* ilist;
  const int* numneigh;
  const int* const* firstneigh;
} b200dp_nlist;

typedef struct b200dp_engine b200dp_engine;

/* Options with their defaults (mixed precision, device 0).  No single
 * counterpart: the reference takes the device from DeepPot::init's gpu_rank
 * and its precision settings from its engine configuration
 * (config/engine.production.json.in). */
void b200dp_options_default(b200dp_options* opt);

/* Loads a model file and prepares device-resident weights.  Replaces
 * DeepPot::init (components/deepmd-op/overlays/api_cc/include/DeepPot.h:475)
 * with the PT-expt backend's load and priming
 * (components/deepmd-op/overlays/api_cc/src/DeepPotPTExpt.cc:324). */
b200dp_status b200dp_create(const char* model_path, const b200dp_options* opt, b200dp_engine** out);
/* Releases the engine's device memory and streams (DeePMD's ~DeepPot,
 * DeepPot.h:457). */
void b200dp_destroy(b200dp_engine* engine);
/* Message of the engine's last failed call: the text that the reference's
 * translate_error (DeepPotPTExpt.cc:295) puts into the exception it throws. */
const char* b200dp_last_error(const b200dp_engine* engine);
/* Model shape: DeepPotPTExpt::cutoff() / numb_types()
 * (components/deepmd-op/overlays/api_cc/include/DeepPotPTExpt.h:103-110),
 * plus the sel and network widths the caller's buffers depend on. */
b200dp_status b200dp_model_info_get(const b200dp_engine* engine, b200dp_model_info* out);
/* CUDA device ordinal the engine runs on (-1 for NULL). */
int b200dp_engine_device(const b200dp_engine* engine);

/* Host buffers in and out (synchronous).  nghost == 0 with a box: periodic
 * system, every periodic image is a neighbour candidate.  nghost > 0: atoms
 * [nlocal, nlocal+nghost) are ghosts (LAMMPS convention), no periodic images
 * are generated, and forces / atom virials are returned for all nlocal+nghost
 * atoms so the caller can fold ghost forces back (reverse communication).
 * coord [nall*3], atype [nall], box [9] (rows are cell vectors; may be NULL
 * when nghost > 0).  force [nall*3], virial [9], atom_energy [nlocal] and
 * atom_virial [nall*9] (both optional, may be NULL).
 * A periodic call (nghost == 0, a box) on page-locked host buffers, without
 * neighbour reuse or stage timing, whose atom count, buffer addresses and box
 * repeat the previous call's is recorded once (at its second occurrence) and
 * then replayed as one CUDA graph: the copies in, the evaluation and the copies
 * out, with the buffers' current contents.  Any other call (pageable buffers,
 * ghosts, a new shape or box) runs directly and drops the recording.  Results
 * are the same either way. */
b200dp_status b200dp_compute_host(b200dp_engine* engine, int nlocal, int nghost, const double* coord,
                                  const int* atype, const double* box, double* energy, double* force,
                                  double* virial, double* atom_energy, double* atom_virial);

/* As b200dp_compute_host, with the caller's LAMMPS full neighbour list
 * (indices into [0, nall)); nghost atoms are ghosts.  Mirrors
 * DeepPot::compute(..., nghost, lmp_list, ago)
 * (components/deepmd-op/overlays/api_cc/include/DeepPot.h:605-690), as
 * PairDeepMD::compute calls it
 * (components/lammps-deepmd-plugin/src/pair_deepmd.cpp:356-371). */
b200dp_status b200dp_compute_host_nlist(b200dp_engine* engine, int nlocal, int nghost, const double* coord,
                                        const int* atype, const b200dp_nlist* nlist, double* energy,
                                        double* force, double* virial, double* atom_energy,
                                        double* atom_virial);

/* Device buffers, work enqueued on `stream` (a cudaStream_t; NULL = legacy
 * default stream): DeepPot::compute_canonical_graph_gpu on the pair style's
 * device views and stream
 * (components/deepmd-op/overlays/api_cc/include/DeepPot.h:903-915, called
 * from components/lammps-deepmd-plugin/src/pair_deepmd_kokkos.cpp:702-709),
 * with coordinates in place of the caller's graph (the engine builds its own
 * neighbour list).  No host synchronisation: device-side error counters are
 * read by b200dp_check.  box and region are HOST arrays (9 and 6 doubles):
 * region = {lo_x, lo_y, lo_z, hi_x, hi_y, hi_z} bounds the binning grid in
 * ghost mode (atoms outside it are still handled correctly, only slower); it
 * may be NULL in periodic mode.  The call is capture-safe once a call of the
 * same or larger size has run (buffers only grow outside capture). */
b200dp_status b200dp_compute_device(b200dp_engine* engine, void* stream, int nlocal, int nghost,
                                    const double* d_coord, const int* d_atype, const double* box,
                                    const double* region, double* d_energy, double* d_force,
                                    double* d_virial, double* d_atom_energy, double* d_atom_virial);

/* As b200dp_compute_device for a periodic system (nghost = 0) whose box
 * lives in device memory (no counterpart in the reference's force call; it
 * serves this library's device-resident NPT driver): d_box [9] (rows are
 * cell vectors) is read by the
 * kernels when they run, so a barostat can change it on the device between
 * calls with no host round trip.  The binning grid (cell counts, stencil
 * reach) comes from the host reference box_ref [9] scaled by min_scale
 * (0 < min_scale <= 1): it serves every device box whose cell vectors are
 * at least min_scale times box_ref's; the caller keeps the box in that range
 * (the MD driver re-references at its synchronisation points). */
b200dp_status b200dp_compute_device_dbox(b200dp_engine* engine, void* stream, int nlocal, const double* d_coord,
                                         const int* d_atype, const double* box_ref, double min_scale,
                                         const double* d_box, double* d_energy, double* d_force, double* d_virial);

/* Synchronises the engine's last stream and converts device error counters
 * into a status (B200DP_ERR_SEL_OVERFLOW / _CAPACITY / _BAD_TYPE /
 * _PEER_TIMEOUT): where the reference raises TORCH_CHECK exceptions that
 * translate_error catches
 * (components/deepmd-op/overlays/api_cc/src/DeepPotPTExpt.cc:295). */
b200dp_status b200dp_check(b200dp_engine* engine);

/* Number of neighbour candidates the last call dropped because a type
 * section exceeded sel (synchronises).  No counterpart: DeePMD truncates at
 * sel silently. */
long long b200dp_sel_overflow_count(b200dp_engine* engine);

/* The canonical neighbour list of the last call, copied to host: nlist and
 * image [nlocal*sel_total] (j index or -1; image code ((n0+512)<<20 |
 * (n1+512)<<10 | (n2+512))), rij [nlocal*sel_total*3].  Any pointer may be
 * NULL.  For parity tests and debugging (no counterpart in the reference). */
b200dp_status b200dp_last_nlist(b200dp_engine* engine, int* nlist, int* image, double* rij);

/* Descriptor and its energy gradient of the last call, [nlocal * descriptor_dim]
 * in atom order, widened to fp64 (no counterpart in the reference; for parity
 * tests).  In mixed precision with the tensor-core
 * path this needs an engine created with keep_descriptor = 1 (else
 * B200DP_ERR_INVALID). */
b200dp_status b200dp_last_descriptor(b200dp_engine* engine, double* descriptor, double* grad_descriptor);

/* Per-stage device times of the last call in milliseconds (CUDA events on
 * the launch stream; the reference's profile families,
 * data/profile-families.csv, time the same stages): [0] neighbour build, [1] descriptor forward,
 * [2] fitting, [3] descriptor backward, [4] force/virial assembly.
 * Timing is enabled by b200dp_set_stage_timing(engine, 1). */
b200dp_status b200dp_set_stage_timing(b200dp_engine* engine, int enable);
/* Self-test of the tensor-core (tcgen05) layer (no counterpart in the
 * reference, whose kernels have no tcgen05 path): C[128 x N] = A[128 x K] *
 * B[N x K]^T from host fp32 arrays, bf16 split with 1 or 3 products,
 * operands in K-major or MN-major layout.  K, N multiples of 16, K <= 256,
 * 16 <= N <= 256, 4*K*(128+N) <= 200 KiB.  Synchronous; allocates its own
 * device buffers. */
b200dp_status b200dp_selftest_mma(int K, int N, int a_mn_major, int b_mn_major, int passes, const float* A,
                                  const float* B, float* C);
/* Neighbour-list build that allocates no device memory (no counterpart in the
 * reference; it exists for callers that must not call cudaMalloc while they
 * run, e.g. an MD engine whose memory pool already owns the GPU, or a step
 * loop that cannot afford the device synchronisation cudaMalloc/cudaFree may
 * cause).  Produces the same formatted list as b200dp_compute_device (same
 * arguments meaning; rcut, ntypes and sel[ntypes] given directly, no engine):
 * d_nlist and d_image [nlocal*sum(sel)] int32, d_rij [nlocal*sum(sel)*3] fp64,
 * all caller-owned device buffers.  Scratch lives in one static device array
 * of about 6.5 MiB that every GPU loading the library keeps until exit; it
 * limits nlocal + nghost to 65536 (larger inputs return B200DP_ERR_CAPACITY)
 * and the binning grid to 65536 cells (coarsened automatically).
 * First call on a device: it looks up that array's device address
 * (cudaGetSymbolAddress) with the device current, and under CUDA's lazy
 * module loading (the default since CUDA 12.2) that lookup is what loads the
 * module holding the array, so the array's memory is reserved then, not when
 * the library is opened.  Make that first call (nlocal = nghost = 0 is
 * enough) before the caller's pool reserves the device's memory and before
 * any stream capture; later calls reserve nothing.
 * Every call synchronises `stream` and reads the device's status counters
 * back with a blocking copy before it returns.  All calls share the array, so
 * calls that overlap on the GPU (other streams, other host threads) race.
 * Status: B200DP_ERR_BAD_TYPE / B200DP_ERR_CAPACITY as for the engine.  A type
 * section holding more than sel neighbours keeps its nearest sel (as DeePMD
 * does); *sel_overflow (optional, may be NULL) receives the number of
 * candidates dropped that way, 0 when no row was truncated. */
b200dp_status b200dp_build_nlist_noalloc(void* stream, int nlocal, int nghost, const double* d_coord,
                                         const int* d_atype, const double* box, const double* region, double rcut,
                                         int ntypes, const int* sel, int* d_nlist, int* d_image, double* d_rij,
                                         long long* sel_overflow);
/* Engine and CUDA stream used by b200dp_direct_energy_force (process-wide;
 * the reference's counterpart is the direct-engine cache primed at model load,
 * components/deepmd-op/overlays/op/pt/dpa4c/graph_compress.cu:1451-1476).
 * NULL engine unbinds. */
b200dp_status b200dp_direct_bind(b200dp_engine* engine, void* stream);

/* Replaces extern "C" dpa_direct_energy_force
 * (components/deepmd-op/overlays/op/pt/dpa4c/graph_compress.cu:1817-1902),
 * called from DeepPotPTExpt::compute_canonical_graph_gpu
 * (components/deepmd-op/overlays/api_cc/src/DeepPotPTExpt.cc:2893-2907).
 * Device pointers, canonical destination-major graph of node_count nodes:
 * atype [node_count] int64; row_ptr [node_count + 1] int64, node i's edges are
 * [row_ptr[i], row_ptr[i+1]); source [edge_storage] uint32 neighbour node;
 * edge_vec [edge_storage][3] fp32, x_source - x_node in Angstrom (periodic
 * images are separate edges).  Outputs are overwritten: energy_out
 * [nloc] per-atom energies, force_out [node_count][3], virial_out
 * [node_count][9] per-atom virials (fp64).  Runs on the bound stream without
 * synchronising; device-side errors are reported by b200dp_check.  Returns 1
 * when handled, 0 when the caller must run its fallback: no engine bound,
 * nloc != node_count (ghost nodes), node_count <= 0, a null pointer, or a
 * launch failure (message in b200dp_last_error of the bound engine). */
int b200dp_direct_energy_force(const int64_t* atype, const int64_t* row_ptr, const uint32_t* source,
                               const float* edge_vec, int64_t node_count, int64_t nloc, int64_t edge_storage,
                               double* energy_out, double* force_out, double* virial_out);

/* Companions of the direct entry, as the LAMMPS Kokkos graph builder and pair
 * style resolve them (components/lammps-deepmd-plugin/src/
 * compact_canonical_graph_kokkos.h:280-300, 825-845; pair_deepmd_kokkos.cpp:
 * 640-665, 725-745):
 *   b200dp_direct_destination_only_ready  1 when an engine is bound and the
 *     call would be handled (node_count > 0, nloc == node_count): the builder
 *     may then omit the source-major CSR (replaces
 *     dpa_direct_destination_only_ready, graph_compress.cu:1804-1815);
 *   b200dp_bind_direct_neighbor_view / b200dp_get_direct_neighbor_view  the
 *     raw-neighbour view (same fields as DpaDirectNeighborView,
 *     direct_neighbor_view.h:1-14): positions x (component c of atom a at
 *     x[a * stride_atom + c * stride_xyz]), model node -> atom, per edge the
 *     candidate atom (ghost images included) and the graph's source array.  While
 *     a view is bound whose source pointer and node count match the call, the
 *     direct entry recomputes every edge vector in fp64 as
 *     (x[candidate] - x[model_to_atom[node]]) * inverse_distance_unit and keeps
 *     the edges within the model's cutoff (so the graph may carry skin
 *     candidates); a null view unbinds;
 *   b200dp_direct_set_need_virial  need_virial & 3 == 0: the next direct calls
 *     leave virial_out untouched and skip the per-atom virial (replaces
 *     dpa_chain_set_need_virial_stream, src/entry/chain_entry.cu:29-41; read at
 *     call time, so a captured graph keeps the request it was captured with);
 *   b200dp_direct_fp32_global_virial_pointer  device pointer to the 9-float
 *     global virial of the last direct call, stable across calls (replaces
 *     dpa_direct_fp32_global_virial_pointer, graph_compress.cu:1512-1517). */
typedef struct b200dp_neighbor_view {
  const double* x;
  const int* model_to_atom;
  const int* candidate_atom;
  const uint32_t* source;
  int64_t stride_atom, stride_xyz, node_count;
  double cutoff_squared, inverse_distance_unit;
} b200dp_neighbor_view;
int b200dp_direct_destination_only_ready(int64_t node_count, int64_t nloc);
void b200dp_bind_direct_neighbor_view(const b200dp_neighbor_view* view);
b200dp_neighbor_view b200dp_get_direct_neighbor_view(void);
void b200dp_direct_set_need_virial(int need_virial, void* stream);
const float* b200dp_direct_fp32_global_virial_pointer(void);

/* ------------------------------------------------------------------ MD
 * Molecular-dynamics driver around an engine (metal units: Angstrom, ps,
 * g/mol, eV, K, bar).  Velocity Verlet (NVE), with a Nose-Hoover chain
 * thermostat (NVT), or with the thermostat and an isotropic
 * Martyna-Tobias-Klein barostat with its own chain (NPT, orthorhombic box
 * scaled about the origin), in the integration order of LAMMPS'
 * fix nve / fix nvt / fix npt iso, which drives the reference's force call
 * (components/lammps/overlays/src/KOKKOS/fix_nh_kokkos.cpp:863-1001; device
 * chain: components/lammps/overlays/src/KOKKOS/dpa_fast_step_kokkos.h:307-400).
 * Positions, velocities, forces, the chain and barostat state and the NPT
 * box stay on the device; a run enqueues its steps on the driver's stream
 * without host synchronisation (the NPT force call reads the box from device
 * memory), and the host reads the state back only at thermo output,
 * snapshot and restore.
 * The box is periodic; positions are not wrapped (the engine images them). */
typedef enum b200dp_md_ensemble { B200DP_MD_NVE = 0, B200DP_MD_NVT = 1, B200DP_MD_NPT = 2 } b200dp_md_ensemble;

/* Neighbour reuse for periodic calls (nghost == 0, box given) of
 * b200dp_compute_device / b200dp_compute_host: candidate pairs within
 * rcut + skin are built on one call and reused by the following calls, whose
 * neighbour rows are formed from them with the new positions (the rows
 * themselves stay the exact per-type rcut rows).  The candidates are built
 * again at least every `every` calls, and on any call where an atom has moved
 * more than skin / 2 from the positions of the last build -- that check and
 * the rebuild run on the device inside the call, with no host round trip
 * (LAMMPS neigh_modify every N check yes, with the check on every step).
 * every = 0 turns reuse off (the default: every call bins from scratch).
 * Replaces the LAMMPS skin neighbour list and its rebuild decision
 * (LO/KOKKOS/npair_kokkos.cpp:151-460; neighbor->decide()). */
b200dp_status b200dp_set_neighbor_reuse(b200dp_engine* engine, double skin, int every);
/* builds[0] = scheduled candidate builds, builds[1] = builds triggered by the
 * displacement check (synchronises the engine's last stream); the
 * counterpart of the neighbour-list build counts LAMMPS reports at the end of
 * a run. */
b200dp_status b200dp_neighbor_stats(b200dp_engine* engine, long long* builds);

/* Halo exchange and reverse fold for spatial domain decomposition, one
 * process per GPU on NVLink peers, through one device buffer per rank that
 * every other rank maps (CUDA IPC): the owned atoms' positions, published
 * every step, and their fixed-point force accumulator.
 *   b200dp_fold_export   allocates this rank's buffer for `capacity` owned
 *                        atoms (the same capacity on every rank) and writes
 *                        its CUDA IPC handle (64 bytes) to `handle`;
 *   b200dp_fold_connect  opens every other rank's handle (handles: nranks
 *                        x 64 bytes, rank order);
 *   b200dp_fold_origins  d_origin [nghost][2] int: owner rank and owner's
 *                        atom index of every ghost row; d_shift [nghost][3]
 *                        f64 (may be NULL without halo_gather): the periodic
 *                        shift added to the owner's position (device memory);
 *   b200dp_halo_publish  copies the owned positions into this rank's buffer;
 *   b200dp_halo_gather   writes the ghost rows nlocal.. of d_coord from the
 *                        owners' published positions (+ shift) -- only after
 *                        every rank's publish of this step has completed
 *                        (b200dp_peer_reduce with nv = 0 on the stream, or
 *                        a one-element all-reduce of the caller's own);
 *   b200dp_compute_device_fold  the ghost-mode force call: energy and virial
 *                        of the owned atoms' edges as usual; the ghost rows'
 *                        reverse contributions are added into the owners'
 *                        accumulators (128-bit integer atomics over NVLink:
 *                        order-independent sums) and d_force is not complete
 *                        yet;
 *   b200dp_fold_finish   after EVERY rank's compute_device_fold has completed
 *                        (b200dp_peer_reduce of energy and virial, nv = 10,
 *                        or a caller's all-reduce of them, on the same
 *                        stream), writes the owned rows of d_force
 *                        and clears the accumulator.
 * Replaces the pair style's forward and reverse ghost communication
 * (PL/pair_deepmd_kokkos.cpp:931, comm->reverse_comm; LAMMPS comm->forward_comm). */
b200dp_status b200dp_fold_export(b200dp_engine* engine, int capacity, void* handle);
b200dp_status b200dp_fold_connect(b200dp_engine* engine, int nranks, int rank, const void* handles);
b200dp_status b200dp_fold_origins(b200dp_engine* engine, int nghost, const int* d_origin, const double* d_shift);
/* Scales every ghost row's periodic shift per component by ratio[3] (host
 * array), enqueued on `stream`: the box of a barostat changed by that ratio
 * and the plan was not rebuilt. */
b200dp_status b200dp_fold_scale_shifts(b200dp_engine* engine, void* stream, const double* ratio);
b200dp_status b200dp_halo_publish(b200dp_engine* engine, void* stream, int nlocal, const double* d_coord);
b200dp_status b200dp_halo_gather(b200dp_engine* engine, void* stream, int nlocal, int nghost, double* d_coord);
b200dp_status b200dp_compute_device_fold(b200dp_engine* engine, void* stream, int nlocal, int nghost,
                                         const double* d_coord, const int* d_atype, const double* region,
                                         double* d_energy, double* d_force, double* d_virial);
b200dp_status b200dp_fold_finish(b200dp_engine* engine, void* stream, int nlocal, double* d_force);
/* Device-side rendezvous of the ranks through their exported buffers, the
 * per-step synchronisation of the peer path without a collective library:
 * the rank's nv values (device memory, 0 <= nv <= 16) are stored into every
 * rank's buffer over NVLink, then its arrival counter; one warp waits until
 * every rank has arrived at this rendezvous and writes the sum of all ranks'
 * values in rank order to d_out (the same bits on every rank).  nv = 0 is a
 * plain barrier (e.g. between halo_publish and halo_gather); nv = 10 with
 * energy and virial is the reduction ahead of fold_finish.  Enqueued on
 * `stream` without host synchronisation (capturable).  Every rank makes the
 * same sequence of calls.  The wait is bounded by max_polls (<= 0: 2^24 polls
 * of ~0.1 us): on expiry d_out is not written and the next b200dp_check
 * returns B200DP_ERR_PEER_TIMEOUT.  Ranks must be on different GPUs (two
 * kernels of one GPU are not guaranteed to run at the same time). Replaces
 * the MPI all-reduce of energy and virial in the pair style
 * (PL/pair_deepmd_kokkos.cpp:937-993). */
b200dp_status b200dp_peer_reduce(b200dp_engine* engine, void* stream, int nv, const double* d_in, double* d_out,
                                 long long max_polls);

typedef struct b200dp_md_params {
  double dt;        /* time step, ps (default 0.0005) */
  int ensemble;     /* b200dp_md_ensemble */
  int chain;        /* Nose-Hoover chain length (NVT, 1..8, default 3) */
  double t_target;  /* K (NVT) */
  double t_damp;    /* thermostat period, ps (NVT, default 0.05) */
  double t_init;    /* K: > 0 draws seeded Gaussian velocities at this temperature (zero momentum) */
  unsigned long long seed;
  double mass[8];   /* g/mol per atom type */
  double p_target;  /* bar (NPT, isotropic) */
  double p_damp;    /* barostat period, ps (NPT, default 0.5) */
  int pchain;       /* barostat Nose-Hoover chain length (NPT, 1..8, default 3) */
  int rebuild_every; /* neighbour candidates rebuilt at least every this many steps and whenever an atom
                        moved more than skin / 2 (default 10; 0 = every step from scratch) */
  double skin;       /* Angstrom, neighbour skin for the reuse (default 2.0) */
  int reserved[8];
} b200dp_md_params;

typedef struct b200dp_md b200dp_md;

b200dp_status b200dp_md_params_default(b200dp_md_params* params);
/* Host arrays: coord [natoms*3], vel [natoms*3] or NULL (then t_init > 0),
 * atype [natoms], box [9].  Computes the initial forces. */
b200dp_status b200dp_md_create(b200dp_engine* engine, int natoms, const double* coord, const double* vel,
                               const int* atype, const double* box, const b200dp_md_params* params,
                               b200dp_md** out);
/* Enqueues nsteps steps; returns without waiting for them. */
b200dp_status b200dp_md_run(b200dp_md* md, int nsteps);
/* Waits for the driver's stream.  thermo[8]: step, potential energy, kinetic
 * energy, temperature (dof = 3N - 3), conserved energy (potential + kinetic +
 * thermostat), pressure (bar), volume, thermostat energy. */
b200dp_status b200dp_md_thermo(b200dp_md* md, double* thermo);
/* Waits for the driver's stream and copies positions / velocities / forces
 * (host arrays of natoms*3, any may be NULL). */
b200dp_status b200dp_md_state(b200dp_md* md, double* coord, double* vel, double* force);
/* Restart.  A snapshot is the run's complete integrator state (positions,
 * velocities, forces, energy and virial of the last force call, thermostat
 * and barostat chains, box, step) in one device buffer of
 * b200dp_md_snapshot_bytes bytes: b200dp_md_snapshot enqueues the copies on
 * the MD stream (no host synchronisation: the run continues while the buffer
 * is kept in HBM or copied out); b200dp_md_restore puts a snapshot of the
 * same system and integrator settings back (B200DP_ERR_INVALID otherwise),
 * after which b200dp_md_run continues the trajectory -- bitwise with
 * rebuild_every <= 1, within fp64 round-off of the neighbour vectors with
 * skin reuse (the candidates are rebuilt from the restored positions).  The
 * restart file is the snapshot's byte image.  Replaces the reference's
 * device-side restart packing (src/runtime/device_restart.cu). */
b200dp_status b200dp_md_snapshot_bytes(const b200dp_md* md, size_t* bytes);
b200dp_status b200dp_md_snapshot(b200dp_md* md, void* d_buf);
b200dp_status b200dp_md_restore(b200dp_md* md, const void* d_buf);
b200dp_status b200dp_md_write_restart(b200dp_md* md, const char* path);
b200dp_status b200dp_md_read_restart(b200dp_md* md, const char* path);
b200dp_status b200dp_md_destroy(b200dp_md* md);

/* Total kernels this library has launched in the process (all engines).
 * Measurement only (no counterpart in the reference). */
long long b200dp_kernel_launches(void);
/* The five stage times of b200dp_set_stage_timing, in milliseconds. */
b200dp_status b200dp_stage_times(b200dp_engine* engine, float* ms5);

/* ------------------------------------------------------------------ multi-GPU driver (C++)
 * Spatially decomposed force evaluation and NVE / NVT molecular dynamics over
 * the GPUs of one node, one process per GPU, orchestrated in C++ with no
 * Python on the path.  Replaces the LAMMPS Kokkos machinery around the pair
 * style in the reference: atom exchange at reneighbouring
 * (components/lammps/overlays/src/KOKKOS/comm_kokkos.cpp:809-1000), ghost
 * borders and forward / reverse communication
 * (components/lammps-deepmd-plugin/src/pair_deepmd_kokkos.cpp:84-124, 931-993)
 * and fix nvt with its chain on the device
 * (components/lammps/overlays/src/KOKKOS/dpa_fast_step_kokkos.h:307-400).
 * Each rank owns the atoms of its sub-box of an orthorhombic periodic box
 * (grid px x py x pz) plus a ghost shell of width `halo` (>= rcut; rcut +
 * skin for MD).  NCCL carries the setup, the atom migration and the ghost
 * plan (host side, at creation and every rebuild_every MD steps); every step
 * runs on the device without host synchronisation: positions published into
 * the ranks' exported buffers, a device-side rendezvous, the ghost gather
 * over NVLink, the force call adding ghost contributions into the owners'
 * fixed-point accumulators, a rendezvous summing energy and virial in rank
 * order, the owners' conversion.  Ranks must be on different GPUs that are
 * NVLink peers.  The engine is the rank's own b200dp_engine (its exported
 * buffer is created here). */
typedef struct b200dp_dd b200dp_dd;
typedef struct b200dp_dd_params {
  int grid[3];         /* ranks along x, y, z (product = number of ranks) */
  double halo;         /* ghost shell width, Angstrom (default 8) */
  long long max_polls; /* bound of every device-side wait (<= 0: the default of b200dp_peer_reduce) */
  int capacity;        /* owned atoms a rank may hold (<= 0: 1.5 x the largest initial count + 1024) */
  int reserved[9];
} b200dp_dd_params;
void b200dp_dd_params_default(b200dp_dd_params* params);
/* 128 bytes that identify one group of ranks (ncclGetUniqueId); rank 0 makes
 * it and the caller hands it to every rank (any host channel). */
b200dp_status b200dp_dd_unique_id(void* id);
/* Collective over the ranks.  Every rank passes the whole system (host
 * arrays: coord [natoms*3], atype [natoms], box [9]) and keeps the atoms whose
 * wrapped position lies in its sub-box; an atom's global index is its id. */
b200dp_status b200dp_dd_create(b200dp_engine* engine, const void* id, int nranks, int rank, const double* box,
                               const b200dp_dd_params* params, int natoms, const double* coord, const int* atype,
                               b200dp_dd** out);
void b200dp_dd_destroy(b200dp_dd* dd);
const char* b200dp_dd_last_error(const b200dp_dd* dd);
/* The driver's CUDA stream (work of the calls below runs on it unless a stream is given). */
void* b200dp_dd_stream(b200dp_dd* dd);
b200dp_status b200dp_dd_counts(b200dp_dd* dd, int* nowned, int* nghost);
/* One decomposed force call on the current positions, enqueued on `stream`
 * (NULL: the driver's), no host synchronisation (capturable).  Every rank
 * calls it the same number of times. */
b200dp_status b200dp_dd_force(b200dp_dd* dd, void* stream);
/* Waits for `stream` and reports the global energy and virial [9] of the last
 * force call (device error counters checked). */
b200dp_status b200dp_dd_result(b200dp_dd* dd, void* stream, double* energy, double* virial);
/* Host copies of the owned atoms (any pointer may be NULL): global ids
 * [nowned], positions, velocities and forces [nowned*3] (synchronises). */
b200dp_status b200dp_dd_owned(b200dp_dd* dd, long long* ids, double* coord, double* vel, double* force);
/* Asynchronous copies on `stream`: new positions of the owned atoms (same
 * atoms and order as b200dp_dd_owned) from host memory, and the owned
 * forces [nowned*3] and the global energy + virial [10] to host memory. */
b200dp_status b200dp_dd_set_positions(b200dp_dd* dd, void* stream, const double* coord);
b200dp_status b200dp_dd_get_forces(b200dp_dd* dd, void* stream, double* force, double* energy_virial);
/* MD over the decomposition: velocity Verlet (NVE) or with the Nose-Hoover
 * chain (NVT), in the order of the single-GPU driver; the global kinetic
 * energy is a device-side rendezvous sum.  vel: global velocities
 * [natoms*3], or NULL for the seeded draw at t_init (the same draw as the
 * single-GPU driver).  Atoms migrate and the ghost plan is rebuilt every
 * rebuild_every steps (0 or 1: every step), between the first half-step and
 * the force call; halo must exceed rcut by twice the largest displacement
 * between rebuilds (checked by b200dp_dd_md_thermo).  NPT (isotropic, fix
 * npt iso order as b200dp_md_*): the barostat and thermostat scalars run on
 * every rank's host from the rendezvous' global kinetic energy and virial (one
 * host read per step); the box, the sub-boxes and the ghost shifts scale with
 * the barostat between plan rebuilds. */
b200dp_status b200dp_dd_md_start(b200dp_dd* dd, const b200dp_md_params* params, const double* vel);
b200dp_status b200dp_dd_md_run(b200dp_dd* dd, int nsteps);
/* Global thermodynamic state, as b200dp_md_thermo. */
b200dp_status b200dp_dd_md_thermo(b200dp_dd* dd, double* thermo);
/* Check of the host plan without GPUs: nranks threads stand in for the
 * ranks.  The atoms are distributed by position; with disp [natoms*3] they
 * are then displaced and migrated to their new owners.  Outputs, rank after
 * rank: owned_ids [natoms] and owned_count [nranks]; ghost_ids, ghost_x /
 * ghost_shift [.*3], ghost_origin [.*2] (owner rank, owner's row) up to
 * ghost_cap rows, ghost_count [nranks] (B200DP_ERR_CAPACITY if the ghosts
 * exceed ghost_cap). */
b200dp_status b200dp_dd_plan_emulate(int nranks, const int* grid, const double* box, double halo, int natoms,
                                     const double* coord, const double* disp, long long* owned_ids,
                                     int* owned_count, long long* ghost_ids, double* ghost_x, double* ghost_shift,
                                     int* ghost_origin, int* ghost_count, int ghost_cap);

#ifdef __cplusplus
}
#endif

#endif /* B200DP_H */
