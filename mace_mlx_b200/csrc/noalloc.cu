// Allocation-free variant of the GPU neighbour-list build.
//
// Some callers cannot allocate device memory at all: an MD engine or a host
// framework that owns every byte of the GPU through its own pool and forbids
// foreign cudaMalloc calls, or a latency-critical loop that cannot afford the
// implicit device synchronisation of cudaMalloc/cudaFree.  They also cannot
// hold a mace_ctx, whose workspace is allocated by mace_ctx_reserve.  For them
// mace_nl_build_noalloc takes only the inputs and caller-owned outputs; its
// scratch (per-atom counts, graph ids, wrap offsets, the scan's temporary
// storage, the inverse cell, the largest graph's size and an error flag) lives
// in one file-scope __device__ array of MACE_NOALLOC_SCRATCH_BYTES, which every
// GPU that loads this library holds until the process exits.
//
// The host cannot use the array's name as a device address (in host code it
// names a host-side shadow), so this file asks the runtime for the device
// address with cudaGetSymbolAddress, with the device current, and caches it
// per device together with the CUDA context it was looked up in; a call that
// finds another context current (the primary context was reset and
// recreated) looks the address up again.  With CUDA's default lazy module
// loading the module holding the array, and so its 4 MiB, is loaded at the
// first lookup on a device: a host that sizes its own pool to all free memory
// should make one call (or set CUDA_MODULE_LOADING=EAGER) before it does so,
// and the first call on each device should come before any stream capture.
// All calls share the one array and it keeps the previous call's contents:
// everything that must start at zero is cleared on every call, and calls that
// overlap on the GPU (different streams, or different host threads on the
// same device) race on the scratch.
//
// Cost: this entry point always uses the all-pairs kernels (one CTA per
// receiver scanning every atom of its graph and every periodic image, twice),
// O(n_g^2 x images) per graph of n_g atoms, because the cell-list build needs
// a per-edge key buffer that a fixed array cannot hold.  Graphs are therefore
// limited to MACE_NOALLOC_MAX_GRAPH_ATOMS atoms each (many small graphs up to
// MACE_NOALLOC_MAX_ATOMS in total are fine); larger single structures belong
// to mace_nl_build, which switches to cell lists.
#include <cmath>
#include <mutex>

#include "common.cuh"

namespace mace {
namespace {

constexpr size_t kScratchBytes = MACE_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) unsigned char g_nl_scratch[kScratchBytes];

std::mutex g_addr_mu;
struct ScratchAddr {
  void* ctx = nullptr;   // CUcontext the address belongs to
  void* addr = nullptr;  // device address of g_nl_scratch in that context
};
ScratchAddr g_addr[64];

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// cuCtxGetCurrent through the runtime's driver entry point (the library does
// not link libcuda itself)
using CtxGetCurrentFn = int (*)(void**);
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      f = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(f);
  }();
  return fn;
}

// device address of the scratch array on the current device and context
int scratch_address(void** out) {
  int dev = -1;
  MACE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(MACE_ERR_BAD_ARG, "device index out of range for the no-alloc scratch");
  CtxGetCurrentFn get = ctx_get_current();
  void* ctx = nullptr;
  if (get && get(&ctx) != 0) ctx = nullptr;
  std::lock_guard<std::mutex> lk(g_addr_mu);
  ScratchAddr& a = g_addr[dev];
  if (!a.addr || !ctx || a.ctx != ctx || !get) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_nl_scratch);
    if (e == cudaErrorMemoryAllocation)
      return fail(MACE_ERR_CUDA, "mace_nl_build_noalloc: loading its 4 MiB static scratch failed: the device is "
                                 "out of memory (make the first call before a memory pool takes all of it)");
    if (e != cudaSuccess || p == nullptr)
      return fail(MACE_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch): ") + cudaGetErrorString(e));
    void* now = nullptr;  // the lookup made the device's context current
    if (get && get(&now) != 0) now = nullptr;
    a.addr = p;
    a.ctx = now;
  }
  *out = a.addr;
  return MACE_OK;
}

// largest graph of graph_ptr (num_graphs + 1 offsets) into *out
__global__ void k_max_graph(const int32_t* __restrict__ graph_ptr, int32_t num_graphs, int32_t* out) {
  int32_t m = 0;
  for (int32_t g = threadIdx.x; g < num_graphs; g += blockDim.x) {
    const int32_t sz = graph_ptr[g + 1] - graph_ptr[g];
    m = sz > m ? sz : m;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const int32_t v = __shfl_xor_sync(0xffffffffu, m, o);
    m = v > m ? v : m;
  }
  __shared__ int32_t warp_max[32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) m = warp_max[w] > m ? warp_max[w] : m;
    *out = m;
  }
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
  // scratch layout: count (n+1) | node graph (n) | wrap (3n) | inverse cell (9 f64) | error flag |
  // largest graph | scan temp
  const size_t scan_bytes = scan_tmp_bytes(n);
  const size_t o_count = 0;
  const size_t o_graph = o_count + align256(sizeof(int32_t) * (n + 1));
  const size_t o_wrap = o_graph + align256(sizeof(int32_t) * n);
  const size_t o_inv = o_wrap + align256(sizeof(int32_t) * 3 * n);
  const size_t o_err = o_inv + align256(sizeof(double) * 9);
  const size_t o_gmax = o_err + align256(sizeof(int));
  const size_t o_scan = o_gmax + align256(sizeof(int32_t));
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
  int32_t* d_gmax = reinterpret_cast<int32_t*>(sb + o_gmax);
  void* scan_tmp = sb + o_scan;

  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the all-pairs kernels cost O(n_g^2) per graph: refuse graphs above the per-graph limit
  k_max_graph<<<1, 256, 0, s>>>(graph_ptr, num_graphs, d_gmax);
  MACE_CUDA_TRY(cudaGetLastError());
  int32_t gmax = 0;
  MACE_CUDA_TRY(cudaMemcpyAsync(&gmax, d_gmax, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  if (gmax > MACE_NOALLOC_MAX_GRAPH_ATOMS)
    return fail(MACE_ERR_BAD_ARG, "mace_nl_build_noalloc: a graph of " + std::to_string(gmax) +
                                      " atoms exceeds the per-graph limit of " +
                                      std::to_string(MACE_NOALLOC_MAX_GRAPH_ATOMS) +
                                      " (all-pairs build; use mace_nl_build with a context for cell lists)");
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
