// Neighbour-list build that allocates no device memory.
//
// Some callers cannot call cudaMalloc while they run: an MD engine that has
// already reserved the GPU's memory for its own pool (a Kokkos or caching
// allocator that owns the device), or a step loop where cudaMalloc/cudaFree
// would add an implicit device synchronisation.  For them this file builds the
// same formatted neighbour list as b200dp_compute_device does, with every piece
// of scratch (wrapped coordinates, cell list, per-type counts, error counters)
// carved out of one file-scope device array of fixed size.  Every GPU that
// loads the library holds that array until the process exits.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>

#include "../../include/b200dp.h"
#include "common.cuh"
#include "nlist.cuh"

namespace b200dp {
namespace {

constexpr int kNoAllocMaxAtoms = 65536;  // nlocal + nghost
constexpr int kNoAllocMaxCells = 65536;  // binning grid cells (the grid is coarsened to fit)
constexpr int kNoAllocMaxTypes = kMaxTypes;

// Byte layout of the static scratch (every block 256-byte aligned).
constexpr size_t align256(size_t b) { return (b + 255) / 256 * 256; }
constexpr size_t kOffXw = 0;
constexpr size_t kOffCellOf = kOffXw + align256(sizeof(double) * 3 * kNoAllocMaxAtoms);
constexpr size_t kOffCellCount = kOffCellOf + align256(sizeof(int) * kNoAllocMaxAtoms);
constexpr size_t kOffCellStart = kOffCellCount + align256(sizeof(int) * kNoAllocMaxCells);
constexpr size_t kOffCursor = kOffCellStart + align256(sizeof(int) * (kNoAllocMaxCells + 1));
constexpr size_t kOffCellRec = kOffCursor + align256(sizeof(int) * kNoAllocMaxCells);
constexpr size_t kOffCounts = kOffCellRec + align256(sizeof(CellRec) * kNoAllocMaxAtoms);
constexpr size_t kOffErr = kOffCounts + align256(sizeof(int) * kNoAllocMaxAtoms * kNoAllocMaxTypes);
constexpr size_t kScratchBytes = kOffErr + align256(sizeof(int) * kErrCount);  // about 6.5 MiB

// The scratch itself.  In host code this name is only a stand-in for the
// device symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// Device address of g_noalloc_scratch, looked up once per device.  Host
// threads may race on the first lookup; each finds the same address, and the
// atomic keeps the cache itself free of a data race.
constexpr int kMaxDevices = 64;
std::atomic<void*> g_scratch_ptr[kMaxDevices];

}  // namespace
}  // namespace b200dp

extern "C" b200dp_status b200dp_build_nlist_noalloc(void* stream, int nlocal, int nghost, const double* d_coord,
                                                     const int* d_atype, const double* box, const double* region,
                                                     double rcut, int ntypes, const int* sel, int* d_nlist,
                                                     int* d_image, double* d_rij, long long* sel_overflow) {
  using namespace b200dp;
  const int nall = nlocal + nghost;
  if (sel_overflow) *sel_overflow = 0;
  if (nlocal < 0 || nghost < 0 || ntypes <= 0 || ntypes > kNoAllocMaxTypes || !sel || !(rcut > 0) ||
      (nall > 0 && (!d_coord || !d_atype)) || (nlocal > 0 && (!d_nlist || !d_image || !d_rij))) {
    return B200DP_ERR_INVALID;
  }
  if (nall > kNoAllocMaxAtoms) return B200DP_ERR_CAPACITY;  // beyond the static scratch
  const bool periodic = (box != nullptr) && nghost == 0;
  if (!periodic && !region) return B200DP_ERR_INVALID;
  int selt = 0;
  for (int t = 0; t < ntypes; ++t) {
    if (sel[t] < 0) return B200DP_ERR_INVALID;
    selt += sel[t];
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return B200DP_ERR_CUDA;
  // First call on this device: look up the scratch address with the device
  // current.  Under CUDA's lazy module loading this lookup is also what loads
  // the module holding the array, i.e. the moment its memory is reserved.
  void* sp = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (!sp) {
    if (cudaGetSymbolAddress(&sp, g_noalloc_scratch) != cudaSuccess || !sp) return B200DP_ERR_CUDA;
    g_scratch_ptr[dev].store(sp, std::memory_order_release);
  }
  unsigned char* base = static_cast<unsigned char*>(sp);
  double* xw = reinterpret_cast<double*>(base + kOffXw);
  int* cell_of = reinterpret_cast<int*>(base + kOffCellOf);
  int* cell_count = reinterpret_cast<int*>(base + kOffCellCount);
  int* cell_start = reinterpret_cast<int*>(base + kOffCellStart);
  int* cursor = reinterpret_cast<int*>(base + kOffCursor);
  CellRec* cell_rec = reinterpret_cast<CellRec*>(base + kOffCellRec);
  int* counts = reinterpret_cast<int*>(base + kOffCounts);
  int* err = reinterpret_cast<int*>(base + kOffErr);
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  // Binning grid (host arithmetic only), coarsened to fit the static scratch.
  GridSpec g;
  switch (make_grid(periodic, box, region, rcut, kNoAllocMaxCells, g)) {
    case 0:
      break;
    case 1:
      return B200DP_ERR_INVALID;
    default:
      return B200DP_ERR_UNSUPPORTED;
  }

  FormatSpec f;
  std::memset(&f, 0, sizeof(f));
  f.nloc = nlocal;
  f.nall = nall;
  f.ntypes = ntypes;
  f.selt = selt;
  f.off[0] = 0;
  for (int t = 0; t < ntypes; ++t) {
    f.sel[t] = sel[t];
    f.off[t + 1] = f.off[t] + sel[t];
  }
  f.rc2 = rcut * rcut;
  format_caps(f);
  if (format_smem_bytes(f) > 200 * 1024) return B200DP_ERR_UNSUPPORTED;

  // Calls share the scratch: the counters that must start at zero are cleared here.
  if (cudaMemsetAsync(err, 0, sizeof(int) * kErrCount, st) != cudaSuccess) return B200DP_ERR_CUDA;
  if (nall > 0) {
    if (cudaMemsetAsync(cell_count, 0, sizeof(int) * g.ncells, st) != cudaSuccess ||
        cudaMemsetAsync(cursor, 0, sizeof(int) * g.ncells, st) != cudaSuccess)
      return B200DP_ERR_CUDA;
    launch_bin(st, nall, d_coord, g, xw, cell_of, cell_count);
    launch_exclusive_scan(st, g.ncells, cell_count, cell_start, nullptr);
    launch_fill_cells(st, nall, xw, d_atype, cell_of, cell_start, cursor, cell_rec);
    launch_format(st, f, g, xw, cell_of, cell_start, cell_rec, d_nlist, d_image, d_rij, counts, err);
  }
  if (cudaGetLastError() != cudaSuccess) return B200DP_ERR_CUDA;
  if (cudaStreamSynchronize(st) != cudaSuccess) return B200DP_ERR_CUDA;
  int h[kErrCount] = {0};
  if (cudaMemcpy(h, err, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess) return B200DP_ERR_CUDA;
  if (sel_overflow) *sel_overflow = h[kErrSelOverflow];
  if (h[kErrBadType]) return B200DP_ERR_BAD_TYPE;
  if (h[kErrCandCapacity]) return B200DP_ERR_CAPACITY;
  return B200DP_OK;
}
