// Allocation-free variant of the GPU neighbour-list build.
//
// Some callers cannot allocate device memory at all: an MD engine or a host
// framework that owns every byte of the GPU through its own pool and forbids
// foreign cudaMalloc calls, or a latency-critical loop that cannot afford the
// implicit device synchronisation of cudaMalloc/cudaFree.  They also cannot
// hold a mace_ctx, whose workspace is allocated by mace_ctx_reserve.  For them
// mace_nl_build_noalloc takes only the inputs and caller-owned outputs; its
// scratch (per-atom counts, graph ids, wrap offsets, the scan's temporary
// storage, the inverse cell and an error flag) lives in one file-scope
// __device__ array of MACE_NOALLOC_SCRATCH_BYTES, which every GPU that loads
// this library holds until the process exits.
//
// The host cannot use the array's name as a device address (in host code it
// names a host-side shadow), so on the first call on each device this file
// asks the runtime for the device address with cudaGetSymbolAddress, with that
// device current, and caches it.  That first call should therefore happen
// before any stream capture.  All calls share the one array and it keeps the
// previous call's contents: everything that must start at zero is cleared on
// every call, and calls that overlap on the GPU (different streams, or
// different host threads on the same device) race on the scratch.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace mace {
namespace {

constexpr size_t kScratchBytes = MACE_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_nl_scratch[kScratchBytes];

std::mutex g_addr_mu;
void* g_addr[64] = {};

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// device address of the scratch array on the current device
int scratch_address(void** out) {
  int dev = -1;
  MACE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MACE_ERR_BAD_ARG, "device index out of range for the no-alloc scratch");
  std::lock_guard<std::mutex> lk(g_addr_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_nl_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(MACE_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
    g_addr[dev] = p;
  }
  *out = g_addr[dev];
  return MACE_OK;
}

#define NA_TRY(x)           \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

}  // namespace
}  // namespace mace

using namespace mace;

extern "C" int mace_nl_build_noalloc(const double* pos, const double* cell, const int32_t* pbc,
                                     const int32_t* graph_ptr, int32_t num_graphs, int64_t n, double r_cut,
                                     int32_t* sender, int32_t* receiver, int32_t* shifts, int32_t* row_ptr,
                                     int32_t* rev, int64_t capacity, int64_t* n_edges, void* stream) {
  if (!pos || !pbc || !graph_ptr || !n_edges || !row_ptr) return fail(MACE_ERR_BAD_ARG, "null argument");
  if (n <= 0 || num_graphs <= 0 || !(r_cut > 0)) return fail(MACE_ERR_BAD_ARG, "bad sizes or cutoff");
  if (n > MACE_NOALLOC_MAX_ATOMS)
    return fail(MACE_ERR_BAD_ARG, "mace_nl_build_noalloc: " + std::to_string(n) + " atoms exceed the limit of " +
                                      std::to_string(MACE_NOALLOC_MAX_ATOMS) + " (use mace_nl_build with a context)");
  // scratch layout: count (n+1) | node graph (n) | wrap (3n) | inverse cell (9 f64) | error flag | scan temp
  const size_t scan_bytes = scan_tmp_bytes(n);
  const size_t o_count = 0;
  const size_t o_graph = o_count + align256(sizeof(int32_t) * (n + 1));
  const size_t o_wrap = o_graph + align256(sizeof(int32_t) * n);
  const size_t o_inv = o_wrap + align256(sizeof(int32_t) * 3 * n);
  const size_t o_err = o_inv + align256(sizeof(double) * 9);
  const size_t o_scan = o_err + align256(sizeof(int));
  if (o_scan + scan_bytes > kScratchBytes)
    return fail(MACE_ERR_BAD_ARG, "mace_nl_build_noalloc: system does not fit the static scratch array");
  void* base = nullptr;
  NA_TRY(scratch_address(&base));
  unsigned char* sb = static_cast<unsigned char*>(base);
  int32_t* count = reinterpret_cast<int32_t*>(sb + o_count);
  int32_t* node_graph = reinterpret_cast<int32_t*>(sb + o_graph);
  int32_t* wrap = reinterpret_cast<int32_t*>(sb + o_wrap);
  double* d_inv = reinterpret_cast<double*>(sb + o_inv);
  int* d_err = reinterpret_cast<int*>(sb + o_err);
  void* scan_tmp = sb + o_scan;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  NlParams p{};
  p.n = n;
  p.pos = pos;
  p.cell = cell;
  p.r_cut = r_cut;
  p.graph_ptr = graph_ptr;
  p.num_graphs = num_graphs;
  bool any_pbc = false;
  for (int d = 0; d < 3; ++d) {
    p.pbc[d] = pbc[d] ? 1 : 0;
    any_pbc |= pbc[d] != 0;
  }
  double hc[9] = {0}, inv[9] = {0};
  if (any_pbc) {
    if (!cell) return fail(MACE_ERR_BAD_ARG, "periodic system without a cell");
    MACE_CUDA_TRY(cudaMemcpyAsync(hc, cell, sizeof(hc), cudaMemcpyDeviceToHost, s));
    MACE_CUDA_TRY(cudaStreamSynchronize(s));
    const double det = hc[0] * (hc[4] * hc[8] - hc[5] * hc[7]) - hc[1] * (hc[3] * hc[8] - hc[5] * hc[6]) +
                       hc[2] * (hc[3] * hc[7] - hc[4] * hc[6]);
    if (!(std::fabs(det) > 1e-12)) return fail(MACE_ERR_BAD_ARG, "periodic cell is singular");
    inv[0] = (hc[4] * hc[8] - hc[5] * hc[7]) / det;
    inv[1] = (hc[2] * hc[7] - hc[1] * hc[8]) / det;
    inv[2] = (hc[1] * hc[5] - hc[2] * hc[4]) / det;
    inv[3] = (hc[5] * hc[6] - hc[3] * hc[8]) / det;
    inv[4] = (hc[0] * hc[8] - hc[2] * hc[6]) / det;
    inv[5] = (hc[2] * hc[3] - hc[0] * hc[5]) / det;
    inv[6] = (hc[3] * hc[7] - hc[4] * hc[6]) / det;
    inv[7] = (hc[1] * hc[6] - hc[0] * hc[7]) / det;
    inv[8] = (hc[0] * hc[4] - hc[1] * hc[3]) / det;
    const double vol = std::fabs(det);
    for (int d = 0; d < 3; ++d) {
      const double* a = hc + 3 * ((d + 1) % 3);
      const double* b = hc + 3 * ((d + 2) % 3);
      const double cx = a[1] * b[2] - a[2] * b[1], cy = a[2] * b[0] - a[0] * b[2], cz = a[0] * b[1] - a[1] * b[0];
      p.reach[d] = r_cut / (vol / std::sqrt(cx * cx + cy * cy + cz * cz)) * (1.0 + 1e-9) + 1e-9;
    }
  }
  MACE_CUDA_TRY(cudaMemcpyAsync(d_inv, inv, sizeof(inv), cudaMemcpyHostToDevice, s));
  p.inv_cell = d_inv;
  p.count = count;
  p.row_ptr = row_ptr;
  p.snd = sender;
  p.rcv = receiver;
  p.shifts = shifts;
  p.rev = rev;
  p.err_flag = d_err;
  p.node_graph = node_graph;
  p.wrap = wrap;
  NA_TRY(launch_nl_prep(p, node_graph, wrap, s));
  NA_TRY(launch_nl_count(p, s));
  MACE_CUDA_TRY(cudaMemsetAsync(count + n, 0, sizeof(int32_t), s));
  NA_TRY(scan_counts(count, row_ptr, n, scan_tmp, scan_bytes, s));
  int32_t total = 0;
  MACE_CUDA_TRY(cudaMemcpyAsync(&total, row_ptr + n, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  *n_edges = total;
  if (total > capacity) return fail(MACE_ERR_NL_OVERFLOW, "edge capacity too small");
  if (total > 0 && (!sender || !receiver || !shifts || !rev)) return fail(MACE_ERR_BAD_ARG, "null edge output");
  MACE_CUDA_TRY(cudaMemsetAsync(d_err, 0, sizeof(int), s));
  NA_TRY(launch_nl_fill(p, s));
  NA_TRY(launch_nl_rev(p, total, s));
  int err = 0;
  MACE_CUDA_TRY(cudaMemcpyAsync(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  if (err) return fail(MACE_ERR_EDGES, "neighbour list is not closed under edge reversal");
  return MACE_OK;
}
