// Neighbour-graph builder: cell binning, warp-ballot compacted candidate
// rows, deterministic per-type (r^2, j, image) ordering, and the stable
// partition of centres by type.
//
// Replaces the LAMMPS/Kokkos candidate list and compact canonical graph of
// the reference (LO/KOKKOS/npair_kokkos.cpp:151-460,
// PL/compact_canonical_graph_kokkos.h:235-821) and the per-step exact cutoff
// (P/include/dpa_chain/exact_cut.cuh:10-20).  Output format is DeePMD's
// formatted neighbour list: per centre, sum(sel) slots, type t at offset
// sum(sel[:t]), -1 padding.
#pragma once

#include <cuda_runtime.h>

#include "common.cuh"

namespace b200dp {

struct GridSpec {
  int periodic;     // 1: fractional grid over the periodic cell; 0: open Cartesian grid
  double B[9];      // cell rows (periodic)
  double Binv[9];   // s_d = sum_a x_a Binv[a*3+d]
  double lo[3];     // open grid origin
  double inv_h[3];  // open grid inverse cell size
  int n[3];         // cells per dimension
  int reach[3];     // stencil half-width in cells
  int ncells;
  // stencil cells whose nearest point is beyond the cutoff are skipped: set for
  // periodic orthorhombic boxes held on the host (every wrapped atom lies in its
  // cell's box of widths cw, so the test is exact up to a 1e-6 A margin)
  int prune;
  double cw[3];
  // periodic box read from device memory ([B | Binv], 18 doubles) instead of
  // B / Binv above, when set: the box of a barostat changes on the device
  // between calls; the cell counts and the stencil reach then come from a
  // reference box that the device box may not undercut (see make_grid_dbox)
  const double* dB;
};

// Grid for a periodic box that lives in device memory: cell counts and reach
// from box_ref scaled by min_scale (the smallest box the grid must serve),
// no cell pruning, kernels reading [B | Binv] from dbox.
int make_grid_dbox(const double* box_ref, double min_scale, const double* dbox, double rcut, long long max_cells,
                   GridSpec& g);
// [B | Binv] of a device box (one thread).
void launch_box_setup(cudaStream_t st, const double* d_box, double* d_bb);

// Cell-sorted atom record written by the fill kernel: the wrapped position
// and the atom's index and type, so the list kernel reaches a candidate's
// data with one 32-byte load.
struct __align__(32) CellRec {
  double x, y, z;
  int j, t;
};

// Binning grid: cells at least rcut / kCellsPerCut wide (coarsened until there
// are at most max_cells), stencil reach covering every cell within rcut.
// Returns 0, or 1 for a degenerate box / region, or 2 for a box so narrow
// that the stencil would exceed 31 cells along a cell vector.
constexpr int kCellsPerCut = 2;
int make_grid(bool periodic, const double* box, const double* region, double rcut, long long max_cells, GridSpec& g);

struct FormatSpec {
  int nloc, nall, ntypes, selt;
  int sel[kMaxTypes];
  int off[kMaxTypes + 1];
  // per-type candidate capacity: type t's in-cutoff candidates of one centre
  // occupy [cap_off[t], cap_off[t+1]) of the warp's buffer (set by
  // format_caps; more than that is a capacity error)
  int cap_off[kMaxTypes + 1];
  int cap_max;
  double rc2;
};

// Fills cap_off / cap_max from sel: max(128, 2 sel[t]) rounded up to 32.
void format_caps(FormatSpec& f);

// Host helpers (identical arithmetic to the oracle's cell set-up).
void make_box_inverse(const double* box, double* Binv, double* width);

// Launchers; all enqueue on `st`.  `gate` (optional, device int): the
// kernels do nothing when *gate == 0, so a rebuild can be decided on the
// device without a host round trip.
// lshift (optional, periodic): the integer lattice shift f of each atom's
// wrap, x_wrapped = x - f . cell.
void launch_bin(cudaStream_t st, int nall, const double* coord, const GridSpec& g, double* xw, int* cell_of,
                int* cell_count, int* lshift = nullptr, const int* gate = nullptr);
// Exclusive scan of n ints into out[0..n] (out[n] = total).  scratch holds
// scan_scratch_ints(n) ints; with scratch == nullptr a single block is used.
void launch_exclusive_scan(cudaStream_t st, int n, const int* in, int* out, int* scratch,
                           const int* gate = nullptr);
size_t scan_scratch_ints(int n);
void launch_fill_cells(cudaStream_t st, int nall, const double* xw, const int* atype, const int* cell_of,
                       const int* cell_start, int* cursor, CellRec* cell_rec, const int* gate = nullptr);
size_t format_smem_bytes(const FormatSpec& f);
void launch_format(cudaStream_t st, const FormatSpec& f, const GridSpec& g, const double* xw, const int* cell_of,
                   const int* cell_start, const CellRec* cell_rec, int* nl_j, int* nl_code, double* nl_rij,
                   int* nl_cnt, int* err);
// Neighbour reuse: skin candidates (every (j, image) within rcand of a centre,
// at most capS per centre, built on the grid of a rcand cutoff), and the rows
// formed from them with the current positions x and the build-time lattice
// shifts.  An atom farther than skin / 2 from its build-time position xref
// sets *stale.
void launch_verlet_build(cudaStream_t st, const FormatSpec& f, const GridSpec& g, double rcand, int capS,
                         const double* xw, const int* cell_of, const int* cell_start, const CellRec* cell_rec,
                         int* cand_j, int* cand_code, int* cand_cnt, int* err, const int* gate = nullptr);
// *trig |= (some atom moved more than skin / 2 from xref); *trig_prev = 0.
void launch_skin_check(cudaStream_t st, int n, const double* x, const double* xref, double skin, int* trig,
                       int* trig_prev);
// If *gate: xref = x and ++*count.
void launch_xref_update(cudaStream_t st, int n, const double* x, double* xref, const int* gate,
                        unsigned long long* count);
void launch_format_verlet(cudaStream_t st, const FormatSpec& f, const GridSpec& g, int capS, double skin,
                          const double* x, const int* atype, const int* lshift, const double* xref,
                          const int* cand_j, const int* cand_code, const int* cand_cnt, int* nl_j, int* nl_code,
                          double* nl_rij, int* nl_cnt, int* err, int* stale);
// Formats a caller-provided candidate list (LAMMPS full list in CSR form).
// Formats a canonical destination-major edge graph (fp32 edge vectors) and
// converts the int64 node types to int32 (invalid types become -1).
// Raw-neighbour geometry for the graph formatter: when x is set, edge k of
// row i is (x[cand[k]] - x[m2a[i]]) * unit in fp64 (component c of atom a at
// x[a * sa + c * sx]) instead of the graph's fp32 edge vector; candidates past
// the cutoff are dropped as usual.
struct RawGeometry {
  const double* x = nullptr;
  const int* m2a = nullptr;
  const int* cand = nullptr;
  long long sa = 0, sx = 0;
  double unit = 1.0;
};
void launch_format_graph(cudaStream_t st, const FormatSpec& f, const int64_t* atype64, const int64_t* row_ptr,
                         const uint32_t* source, const float* edge_vec, int* atype32, int* nl_j, int* nl_code,
                         double* nl_rij, int* nl_cnt, int* err, const RawGeometry& raw = RawGeometry{});
void launch_format_candidates(cudaStream_t st, const FormatSpec& f, const double* coord, const int* atype,
                              const int* ilist, const int* cand_start, const int* cand, int* nl_j, int* nl_code,
                              double* nl_rij, int* nl_cnt, int* err);
// Tables over the type-grouped rows that later kernels need, filled by the
// partition's scan (no launches of their own): istart[nnets + 1], the first
// work item of each embedding net (a net's rows are all rows, or its centre
// type's rows when tos == 0; ceil(rows / item_rows) items padded to a multiple
// of item_pad), and ftile[ntypes + 1], the first 128-row fitting tile of each
// type.  Either pointer may be null.
struct RowTables {
  int nnets = 0, tos = 1, item_rows = 8, item_pad = 1;
  int* istart = nullptr;
  int* ftile = nullptr;
};
void launch_type_partition(cudaStream_t st, int nloc, int ntypes, const int* atype, int* blk_counts,
                           int* type_start, int* perm_pos, int* perm_atom, int* err,
                           const RowTables& tables = RowTables{});
size_t type_partition_blocks(int nloc);

}  // namespace b200dp
