// Neighbour list on the GPU with the "ijS" contract of the reference's
// _build_neighbor_list (mace_mlx/calculators.py:40-62; matscipy/ASE):
// every (i, j, S) with |x_j - x_i + S @ cell| < r_cut, except i == j with
// S == 0, S = 0 along non-periodic axes, both directions present.
//
// Candidate images come from wrapped fractional coordinates, but the
// distance test itself is evaluated in float64 on the original positions as
// (x_j - x_i) + S @ cell, the same expression as the CPU oracle, so the edge
// set is bit-exact against it away from exact ties.
//
// Output is sorted by (receiver, sender, S): one CTA per receiver, senders
// handed out in ascending chunks, an ordered block scan for the write offsets.
#include <cub/cub.cuh>

#include "common.cuh"

namespace mace {

namespace {

constexpr int NLT = 256;

__device__ __forceinline__ int graph_of(const int32_t* gp, int ng, int64_t i) {
  int lo = 0, hi = ng - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (gp[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void k_nl_prep(NlParams p, int32_t* node_graph, int32_t* wrap) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  node_graph[i] = graph_of(p.graph_ptr, p.num_graphs, i);
  for (int d = 0; d < 3; ++d) {
    int w = 0;
    if (p.pbc[d]) {
      double f = p.pos[3 * i + 0] * p.inv_cell[0 * 3 + d] + p.pos[3 * i + 1] * p.inv_cell[1 * 3 + d] +
                 p.pos[3 * i + 2] * p.inv_cell[2 * 3 + d];
      w = (int)floor(f);
    }
    wrap[3 * i + d] = w;
  }
}

struct PairIter {
  int lo[3], hi[3];
  int base[3];  // S = S' + base
};

__device__ __forceinline__ PairIter pair_ranges(const NlParams& p, int64_t i, int64_t j) {
  PairIter it;
  for (int d = 0; d < 3; ++d) {
    if (!p.pbc[d]) {
      it.lo[d] = 0;
      it.hi[d] = 0;
      it.base[d] = 0;
      continue;
    }
    // wrapped fractional coordinates
    double fi = p.pos[3 * i + 0] * p.inv_cell[0 * 3 + d] + p.pos[3 * i + 1] * p.inv_cell[1 * 3 + d] +
                p.pos[3 * i + 2] * p.inv_cell[2 * 3 + d] - p.wrap[3 * i + d];
    double fj = p.pos[3 * j + 0] * p.inv_cell[0 * 3 + d] + p.pos[3 * j + 1] * p.inv_cell[1 * 3 + d] +
                p.pos[3 * j + 2] * p.inv_cell[2 * 3 + d] - p.wrap[3 * j + d];
    double df = fj - fi;
    double reach = p.reach[d];
    it.lo[d] = (int)ceil(-reach - df);
    it.hi[d] = (int)floor(reach - df);
    it.base[d] = p.wrap[3 * i + d] - p.wrap[3 * j + d];
  }
  return it;
}

__device__ __forceinline__ bool hit(const NlParams& p, int64_t i, int64_t j, const int S[3]) {
  if (i == j && S[0] == 0 && S[1] == 0 && S[2] == 0) return false;
  double d2 = 0.0;
  for (int c = 0; c < 3; ++c) {
    double off = 0.0;
    if (p.pbc[0] || p.pbc[1] || p.pbc[2]) {
      off = __dadd_rn(__dadd_rn(__dmul_rn((double)S[0], p.cell[0 * 3 + c]),
                                __dmul_rn((double)S[1], p.cell[1 * 3 + c])),
                      __dmul_rn((double)S[2], p.cell[2 * 3 + c]));
    }
    double dx = __dadd_rn(__dsub_rn(p.pos[3 * j + c], p.pos[3 * i + c]), off);
    d2 = __dadd_rn(d2, __dmul_rn(dx, dx));
  }
  return d2 < p.r_cut * p.r_cut;
}

template <bool WRITE>
__device__ __forceinline__ int pair_hits(const NlParams& p, int64_t i, int64_t j, int64_t out) {
  PairIter it = pair_ranges(p, i, j);
  int cnt = 0;
  for (int a = it.lo[0]; a <= it.hi[0]; ++a)
    for (int b = it.lo[1]; b <= it.hi[1]; ++b)
      for (int c = it.lo[2]; c <= it.hi[2]; ++c) {
        int S[3] = {a + it.base[0], b + it.base[1], c + it.base[2]};
        if (hit(p, i, j, S)) {
          if (WRITE) {
            int64_t o = out + cnt;
            p.snd[o] = (int32_t)i;
            p.rcv[o] = (int32_t)j;
            p.shifts[3 * o + 0] = S[0];
            p.shifts[3 * o + 1] = S[1];
            p.shifts[3 * o + 2] = S[2];
          }
          ++cnt;
        }
      }
  return cnt;
}

__global__ void __launch_bounds__(NLT) k_nl_count(NlParams p) {
  using BR = cub::BlockReduce<int, NLT>;
  __shared__ typename BR::TempStorage tmp;
  const int64_t j = blockIdx.x;
  const int g = p.node_graph[j];
  const int64_t b = p.graph_ptr[g], e = p.graph_ptr[g + 1];
  int cnt = 0;
  for (int64_t i = b + threadIdx.x; i < e; i += NLT) cnt += pair_hits<false>(p, i, j, 0);
  int tot = BR(tmp).Sum(cnt);
  if (threadIdx.x == 0) p.count[j] = tot;
}

__global__ void __launch_bounds__(NLT) k_nl_fill(NlParams p) {
  using BS = cub::BlockScan<int, NLT>;
  __shared__ typename BS::TempStorage tmp;
  __shared__ int64_t s_base;
  const int64_t j = blockIdx.x;
  const int g = p.node_graph[j];
  const int64_t b = p.graph_ptr[g], e = p.graph_ptr[g + 1];
  if (threadIdx.x == 0) s_base = p.row_ptr[j];
  __syncthreads();
  for (int64_t c0 = b; c0 < e; c0 += NLT) {
    const int64_t i = c0 + threadIdx.x;
    int cnt = (i < e) ? pair_hits<false>(p, i, j, 0) : 0;
    int off, tot;
    BS(tmp).ExclusiveSum(cnt, off, tot);
    const int64_t base = s_base;
    if (i < e && cnt) pair_hits<true>(p, i, j, base + off);
    __syncthreads();
    if (threadIdx.x == 0) s_base = base + tot;
    __syncthreads();
  }
}

__device__ __forceinline__ int cmp_edge(const NlParams& p, int64_t e, int snd, const int S[3]) {
  int a = p.snd[e];
  if (a != snd) return a < snd ? -1 : 1;
  for (int d = 0; d < 3; ++d) {
    int v = p.shifts[3 * e + d];
    if (v != S[d]) return v < S[d] ? -1 : 1;
  }
  return 0;
}

__global__ void k_nl_rev(NlParams p, int64_t E) {
  int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= E) return;
  const int i = p.snd[e], j = p.rcv[e];
  const int S[3] = {-p.shifts[3 * e + 0], -p.shifts[3 * e + 1], -p.shifts[3 * e + 2]};
  int64_t lo = p.row_ptr[i], hi = p.row_ptr[i + 1] - 1;
  int64_t found = -1;
  while (lo <= hi) {
    int64_t mid = (lo + hi) >> 1;
    int c = cmp_edge(p, mid, j, S);
    if (c == 0) {
      found = mid;
      break;
    }
    if (c < 0) lo = mid + 1;
    else hi = mid - 1;
  }
  p.rev[e] = (int32_t)found;
  if (found < 0) atomicExch(p.err_flag, 1);
}

// ---------------------------------------------------------------------------
// cell lists (one graph): atoms binned with bins at least one cutoff wide (in
// fractional units, r_cut / plane spacing), so every neighbour of an atom lies
// in the 27 bins around its own; periodic axes wrap, open axes end.  The same
// float64 distance test decides, so the edge set equals the all-pairs one.
// ---------------------------------------------------------------------------
__device__ __forceinline__ double frac_wrapped(const NlParams& p, int64_t i, int d) {
  return p.pos[3 * i + 0] * p.inv_cell[0 * 3 + d] + p.pos[3 * i + 1] * p.inv_cell[1 * 3 + d] +
         p.pos[3 * i + 2] * p.inv_cell[2 * 3 + d] - p.wrap[3 * i + d];
}

__device__ __forceinline__ double bin_space(const NlParams& p, int64_t i, int d) {
  return p.use_frac ? frac_wrapped(p, i, d) : p.pos[3 * i + d];
}

__device__ __forceinline__ int bin_coord(const NlParams& p, int64_t i, int d) {
  const double x = bin_space(p, i, d);
  const double t = p.pbc[d] ? x * p.nbin[d] : (x - p.origin[d]) * p.inv_binw[d];
  const int b = (int)floor(t);
  return b < 0 ? 0 : (b >= p.nbin[d] ? p.nbin[d] - 1 : b);
}

__global__ void k_nl_bin(NlParams p) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const int b = (bin_coord(p, i, 2) * p.nbin[1] + bin_coord(p, i, 1)) * p.nbin[0] + bin_coord(p, i, 0);
  p.atom_bin[i] = b;
  atomicAdd(p.bin_fill + b, 1);
}

__global__ void k_nl_scatter(NlParams p) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= p.n) return;
  const int b = p.atom_bin[i];
  const int slot = atomicAdd(p.bin_fill + b, 1);
  p.bin_atoms[p.bin_start[b] + slot] = (int32_t)i;
}

// Visit every candidate sender of receiver j (lanes of one warp in parallel,
// all 32 lanes in every step): f(valid, i, S) for each (i, S) in the 27
// surrounding bins, S the integer shift of the all-pairs test (image k of the
// bin: S = wrap_i - wrap_j - k); lanes past the end of a bin get valid = false.
template <class F>
__device__ __forceinline__ void cl_candidates(const NlParams& p, int64_t j, int lane, F&& f) {
  int bj[3];
  for (int d = 0; d < 3; ++d) bj[d] = bin_coord(p, j, d);
  for (int dz = -1; dz <= 1; ++dz)
    for (int dy = -1; dy <= 1; ++dy)
      for (int dx = -1; dx <= 1; ++dx) {
        const int dd[3] = {dx, dy, dz};
        int b[3], k[3];
        bool ok = true;
        for (int d = 0; d < 3; ++d) {
          int v = bj[d] + dd[d];
          k[d] = 0;
          if (p.pbc[d]) {
            if (v < 0) { v += p.nbin[d]; k[d] = -1; }
            else if (v >= p.nbin[d]) { v -= p.nbin[d]; k[d] = 1; }
          } else if (v < 0 || v >= p.nbin[d]) {
            ok = false;
          }
          b[d] = v;
        }
        if (!ok) continue;
        const int bin = (b[2] * p.nbin[1] + b[1]) * p.nbin[0] + b[0];
        const int s0 = p.bin_start[bin], s1 = p.bin_start[bin + 1];
        for (int q0 = s0; q0 < s1; q0 += 32) {
          const int q = q0 + lane;
          const bool valid = q < s1;
          const int64_t i = valid ? p.bin_atoms[q] : j;
          int S[3];
          for (int d = 0; d < 3; ++d) S[d] = p.pbc[d] ? p.wrap[3 * i + d] - p.wrap[3 * j + d] - k[d] : 0;
          f(valid, i, S);
        }
      }
}

__global__ void __launch_bounds__(256) k_nl_cl_count(NlParams p) {
  const int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= p.n) return;
  int cnt = 0;
  cl_candidates(p, j, lane, [&](bool valid, int64_t i, const int S[3]) { cnt += (valid && hit(p, i, j, S)) ? 1 : 0; });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
  if (lane == 0) p.count[j] = cnt;
}

__device__ __forceinline__ unsigned long long edge_key(int64_t i, const int S[3]) {
  return ((unsigned long long)i << 30) | ((unsigned long long)(S[0] + 512) << 20) |
         ((unsigned long long)(S[1] + 512) << 10) | (unsigned long long)(S[2] + 512);
}

// hits of receiver j appended unsorted to keys[row_ptr[j]..], then placed in
// (sender, S) order by rank (keys are unique within a receiver)
__global__ void __launch_bounds__(256) k_nl_cl_fill(NlParams p) {
  const int64_t j = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (j >= p.n) return;
  const int64_t base = p.row_ptr[j], end = p.row_ptr[j + 1];
  int64_t cursor = base;
  cl_candidates(p, j, lane, [&](bool valid, int64_t i, const int S[3]) {
    const bool h = valid && hit(p, i, j, S);
    bool in_range = true;
    for (int d = 0; d < 3; ++d) in_range &= (S[d] >= -NL_SHIFT_RANGE && S[d] <= NL_SHIFT_RANGE);
    if (h && !in_range) atomicExch(p.err_flag, NL_ERR_SHIFT);
    const unsigned hits = __ballot_sync(0xffffffffu, h && in_range);
    if (h && in_range) {
      const int64_t o = cursor + __popc(hits & ((1u << lane) - 1));
      if (o < end) p.keys[o] = edge_key(i, S);
    }
    cursor += __popc(hits);
  });
  __syncwarp();
  const int64_t n = end - base;
  for (int64_t a = lane; a < n; a += 32) {
    const unsigned long long ka = p.keys[base + a];
    int64_t rank = 0;
    for (int64_t b = 0; b < n; ++b) rank += p.keys[base + b] < ka ? 1 : 0;
    const int64_t o = base + rank;
    p.snd[o] = (int32_t)(ka >> 30);
    p.rcv[o] = (int32_t)j;
    p.shifts[3 * o + 0] = (int)((ka >> 20) & 1023) - 512;
    p.shifts[3 * o + 1] = (int)((ka >> 10) & 1023) - 512;
    p.shifts[3 * o + 2] = (int)(ka & 1023) - 512;
  }
}

// bounding box of the bin coordinates (fractional with a cell, else Cartesian):
// out6 = (min 0, min 1, min 2, max 0, max 1, max 2)
__global__ void __launch_bounds__(1024) k_nl_bbox(NlParams p, double* out6) {
  __shared__ double red[6][32];
  double lo[3] = {1e300, 1e300, 1e300}, hi[3] = {-1e300, -1e300, -1e300};
  for (int64_t i = threadIdx.x; i < p.n; i += blockDim.x)
    for (int d = 0; d < 3; ++d) {
      const double x = bin_space(p, i, d);
      lo[d] = fmin(lo[d], x);
      hi[d] = fmax(hi[d], x);
    }
  for (int o = 16; o > 0; o >>= 1)
    for (int d = 0; d < 3; ++d) {
      lo[d] = fmin(lo[d], __shfl_xor_sync(0xffffffffu, lo[d], o));
      hi[d] = fmax(hi[d], __shfl_xor_sync(0xffffffffu, hi[d], o));
    }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0)
    for (int d = 0; d < 3; ++d) {
      red[d][w] = lo[d];
      red[3 + d][w] = hi[d];
    }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int d = 0; d < 3; ++d) {
      double a = red[d][0], b = red[3 + d][0];
      for (int q = 1; q < (int)(blockDim.x >> 5); ++q) {
        a = fmin(a, red[d][q]);
        b = fmax(b, red[3 + d][q]);
      }
      out6[d] = a;
      out6[3 + d] = b;
    }
  }
}

}  // namespace

int launch_nl_bins(const NlParams& p, void* tmp, size_t tmp_bytes, cudaStream_t s) {
  const int nb = p.nbin[0] * p.nbin[1] * p.nbin[2];
  MACE_CUDA_TRY(cudaMemsetAsync(p.bin_fill, 0, sizeof(int32_t) * (nb + 1), s));
  const unsigned g = (unsigned)((p.n + 255) / 256);
  k_nl_bin<<<g, 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("nl_bin");
  MACE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, p.bin_fill, p.bin_start, nb + 1, s));
  MACE_CUDA_TRY(cudaMemsetAsync(p.bin_fill, 0, sizeof(int32_t) * nb, s));
  k_nl_scatter<<<g, 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("nl_scatter");
  return MACE_OK;
}

int launch_nl_cl_count(const NlParams& p, cudaStream_t s) {
  if (p.n == 0) return MACE_OK;
  k_nl_cl_count<<<(unsigned)((p.n * 32 + 255) / 256), 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("nl_cl_count");
  return MACE_OK;
}

int launch_nl_cl_fill(const NlParams& p, cudaStream_t s) {
  if (p.n == 0) return MACE_OK;
  k_nl_cl_fill<<<(unsigned)((p.n * 32 + 255) / 256), 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("nl_cl_fill");
  return MACE_OK;
}

int launch_nl_bbox(const NlParams& p, double* out6, cudaStream_t s) {
  k_nl_bbox<<<1, 1024, 0, s>>>(p, out6);
  MACE_LAUNCH_CHECK("nl_bbox");
  return MACE_OK;
}

int launch_nl_prep(const NlParams& p, int32_t* node_graph, int32_t* wrap, cudaStream_t s) {
  if (p.n == 0) return MACE_OK;
  k_nl_prep<<<(unsigned)((p.n + 255) / 256), 256, 0, s>>>(p, node_graph, wrap);
  MACE_LAUNCH_CHECK("nl_prep");
  return MACE_OK;
}

int launch_nl_count(const NlParams& p, cudaStream_t s) {
  if (p.n == 0) return MACE_OK;
  k_nl_count<<<(unsigned)p.n, NLT, 0, s>>>(p);
  MACE_LAUNCH_CHECK("nl_count");
  return MACE_OK;
}

int launch_nl_fill(const NlParams& p, cudaStream_t s) {
  if (p.n == 0) return MACE_OK;
  k_nl_fill<<<(unsigned)p.n, NLT, 0, s>>>(p);
  MACE_LAUNCH_CHECK("nl_fill");
  return MACE_OK;
}

int launch_nl_rev(const NlParams& p, int64_t E, cudaStream_t s) {
  if (E == 0) return MACE_OK;
  k_nl_rev<<<(unsigned)((E + 255) / 256), 256, 0, s>>>(p, E);
  MACE_LAUNCH_CHECK("nl_rev");
  return MACE_OK;
}

size_t scan_tmp_bytes(int64_t n) {
  size_t bytes = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, bytes, (int32_t*)nullptr, (int32_t*)nullptr, (int)(n + 1));
  return bytes;
}

int scan_counts(int32_t* count, int32_t* row_ptr, int64_t n, void* tmp, size_t tmp_bytes,
                cudaStream_t s) {
  MACE_CUDA_TRY(cub::DeviceScan::ExclusiveSum(tmp, tmp_bytes, count, row_ptr, (int)(n + 1), s));
  return MACE_OK;
}

}  // namespace mace
