// Node linears (o3.Linear, the skip_tp's species-indexed channel mixing and
// their transposes) on the 5th-generation tensor cores.
//
// A job maps rows (node, m) of its concat-K input slots to one output slot:
//   out[n, out_off + m C + o] (+)= alpha * sum_k in[n, k_off[k/C] + m C + k%C] W[k][o].
// One CTA computes a tile of TN = floor(128 / d) whole nodes (TN d <= 128 rows)
// times NC output columns (column group g of C / NC) in TMEM, over 32-wide K
// chunks t:
//   D_small += A_lo B_hi + A_hi B_lo,   D_big[t & 1] += A_hi B_hi
// (kind::tf32, 4 K-steps of 8) with A the 128 x 32 input chunk and B the
// weight chunk (NC rows x 32, the transpose of W's 32 rows); hi = x rounded to
// tf32, lo = (x - hi) rounded to tf32 (the 3xTF32 split), and the epilogue
// adds the three accumulators in fp32.  The tensor core truncates when it
// accumulates, and the error grows with the number of accumulation steps into
// one accumulator: the small terms in their own accumulator and two
// alternating big ones keep it near fp32 rounding.
//
// Data movement: the input chunk of a tile is one TMA box of a 3-D tensor map
// over the input slot ({C floats, d rows m, N nodes}, box {32, d, TN},
// 128-byte swizzle, so it lands in the MMA's K-major SW128 layout; nodes past
// N read as zeros), and the weights never change, so their operand images
// (tf32 hi and lo, 128B-swizzled K-major, made once per context by
// k_tc_image) arrive as two bulk copies per chunk.  One thread keeps NST
// chunks in flight; the four converter warps turn each landed chunk into its
// hi part (in place) and lo part, an elementwise pass over the 16 KB tile, so
// global-memory latency is covered by the stage depth rather than by
// registers.  Small launches split the output columns into groups (NC = C/2
// or C/4) so that the row tiles of one launch still reach every SM.
//
// Species-indexed jobs (the skip connection) run one pass per distinct
// species in the tile, with the rows of other species zeroed in A and that
// species' weight image in B.
//
// Every mbarrier wait is bounded (about 2 s).  A wait that gives up makes the
// whole CTA leave the K loop (agreed through __syncthreads_or), wait (bounded)
// for its MMAs and copies, record TC_ERR_TIMEOUT in the error flag, free its
// TMEM and return.
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "tc.cuh"

namespace mace {

namespace {

constexpr int TL_ROWS = 128;
constexpr int TL_THREADS = 192;  // warps 0-3: hi/lo conversion + epilogue; 4: copies; 5: MMAs
constexpr int TL_MAX_MAPS = 32;  // (job, input slot) tensor maps per launch

// operand stages that fit 227 KB next to one 128-row A tile pair each
__host__ __device__ constexpr int tl_stages(int NC) { return NC >= 96 ? 3 : (NC == 64 ? 4 : 5); }

template <int NC>
__host__ __device__ constexpr uint32_t tl_tmem_cols() {
  return 3 * NC <= 128 ? 128 : (3 * NC <= 256 ? 256 : 512);
}

template <int NC>
struct TlSmem {
  static constexpr int NST = tl_stages(NC);
  static constexpr int A = TL_ROWS * 128;  // one 128-row x 32 fp32 operand tile
  static constexpr int B = NC * 128;       // one NC-row x 32 operand tile
  static constexpr int STAGE = 2 * A + 2 * B;  // A hi (TMA target, converted in place), A lo, B hi, B lo
  static constexpr int BYTES = NST * STAGE + 1024;  // + alignment slack
};

struct alignas(64) LinTcParams {
  CUtensorMap map[TL_MAX_MAPS];    // per (job, input slot): dims {C, d, N}, box {32, d, tn}
  LinParams p;
  int tile_start[MACE_MAX_MID + 1];  // first row tile of each job; [n_jobs] = total
  int map_base[MACE_MAX_MID];        // first tensor map of each job
  int tn[MACE_MAX_MID];              // nodes per row tile of each job
  int cs;                            // column groups per row tile (C / NC)
};

template <int NC>
__global__ void __launch_bounds__(TL_THREADS, 1) k_linear_tc(const __grid_constant__ LinTcParams q) {
  using S = TlSmem<NC>;
  constexpr int NST = S::NST;
  extern __shared__ uint8_t smem_raw[];
  // full[s] (A box and weight chunk landed), ready[s] (hi/lo stored), free[s] (MMAs done), done
  __shared__ __align__(8) uint64_t bars[3 * NST + 1];
  __shared__ uint32_t tslot;
  __shared__ int abort_flag;
  __shared__ uint32_t zmask[8];
  __shared__ int sZ[TL_ROWS + 1];
  const LinParams& p = q.p;
  const int item = blockIdx.x / q.cs, g = blockIdx.x - item * q.cs;
  int jx = 0;
  while (jx + 1 < p.n_jobs && q.tile_start[jx + 1] <= item) ++jx;
  const LinJob& jb = p.job[jx];
  const int C = p.C;
  const int d = jb.d, TN = q.tn[jx];
  const int rows_tile = TN * d;
  const int64_t node0 = (int64_t)(item - q.tile_start[jx]) * TN;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t base = (tc::smem_u32(smem_raw) + 1023u) & ~1023u;
  auto FULL = [&](int s) { return tc::smem_u32(&bars[s]); };
  auto READY = [&](int s) { return tc::smem_u32(&bars[NST + s]); };
  auto FREE = [&](int s) { return tc::smem_u32(&bars[2 * NST + s]); };
  const uint32_t DONE = tc::smem_u32(&bars[3 * NST]);
  volatile int* abort = &abort_flag;

  const int nck = C / 32;
  const int nchunks = jb.n_k * nck;
  const int64_t zimg = (int64_t)nchunks * 2 * C * 32;  // floats of one species' image
  const uint32_t abox = (uint32_t)rows_tile * 128;     // bytes of one A box
  int issued = 0;  // chunk copies issued (warp 4, lane 0)
  // one chunk's copies into stage t % NST: the A box, then the weight chunk's hi and lo rows of column group g
  auto issue = [&](int t, int z) {
    const int s = t % NST;
    const int tt = t % nchunks;
    const int ks = tt / nck, kc = tt - ks * nck;
    const uint32_t st = base + s * S::STAGE;
    tc::mbar_expect_tx(FULL(s), abox + 2 * S::B);
    tc::tma_load3(st, &q.map[q.map_base[jx] + ks], 32 * kc, 0, (int)node0, FULL(s));
    const float* img = jb.tc + z * zimg + (int64_t)tt * 2 * C * 32 + (int64_t)g * NC * 32;
    tc::bulk_g2s(st + 2 * S::A, img, S::B, FULL(s));
    tc::bulk_g2s(st + 2 * S::A + S::B, img + C * 32, S::B, FULL(s));
  };

  if (warp == 4 && lane == 0) {
    tc::prefetch_tensormap(&q.map[q.map_base[jx]]);
    for (int s = 0; s < NST; ++s) {
      tc::mbar_init(FULL(s), 1);
      tc::mbar_init(READY(s), 128);
      tc::mbar_init(FREE(s), 1);
    }
    tc::mbar_init(DONE, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
    // without species passes the first chunks do not wait for the tile set-up
    if (!jb.species)
      for (; issued < NST && issued < nchunks; ++issued) issue(issued, 0);
  }
  if (warp == 0) {
    tc::tmem_alloc(tc::smem_u32(&tslot), tl_tmem_cols<NC>());
    tc::tmem_relinquish();
  }
  if (tid < 8) zmask[tid] = 0;
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = tslot;
  // distinct species of the tile's rows, ascending (species-indexed jobs)
  int n_pass = 1;
  if (jb.species) {
    bool wide = false;
    if (tid < TN && node0 + tid < p.N) {
      const int z = jb.species[node0 + tid];
      if (z < 256)
        atomicOr(&zmask[z >> 5], 1u << (z & 31));
      else
        wide = true;
    }
    if (__syncthreads_or(wide)) {  // species index beyond the mask: serial scan
      if (tid == 0) {
        int nd = 0;
        for (int r = 0; r < TN && node0 + r < p.N; ++r) {
          const int z = jb.species[node0 + r];
          bool seen = false;
          for (int k = 0; k < nd && !seen; ++k) seen = sZ[k] == z;
          if (!seen) sZ[nd++] = z;
        }
        sZ[TL_ROWS] = nd;
      }
    } else if (tid == 0) {
      int nd = 0;
      for (int w = 0; w < 8; ++w)
        for (uint32_t m = zmask[w]; m; m &= m - 1) sZ[nd++] = 32 * w + __ffs(m) - 1;
      sZ[TL_ROWS] = nd;
    }
    __syncthreads();
    n_pass = sZ[TL_ROWS];
  }
  const int total = n_pass * nchunks;
  constexpr uint32_t IDESC = tc::idesc_tf32(TL_ROWS, NC);

  if (warp == 4) {
    // ---------------- copies ----------------
    if (lane == 0) {
      for (int t = issued; t < total; ++t) {
        const int s = t % NST, u = t / NST;
        if (t >= NST && !tc::mbar_wait_or_abort(FREE(s), (u - 1) & 1, abort)) break;
        issue(t, jb.species ? sZ[t / nchunks] : 0);
        issued = t + 1;
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMAs ----------------
    if (lane == 0) {
      for (int t = 0; t < total; ++t) {
        const int s = t % NST, u = t / NST;
        if (!tc::mbar_wait_or_abort(READY(s), u & 1, abort)) break;
        tc::fence_after_sync();
        const uint32_t st = base + s * S::STAGE;
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          const uint32_t ah = st + kb * 32, al = ah + S::A;
          const uint32_t bh = st + 2 * S::A + kb * 32, bl = bh + S::B;
          tc::mma_tf32(tmem + 2 * NC, tc::sw128_desc(al), tc::sw128_desc(bh), IDESC, (t > 0 || kb > 0));
          tc::mma_tf32(tmem + 2 * NC, tc::sw128_desc(ah), tc::sw128_desc(bl), IDESC, 1);
          tc::mma_tf32(tmem + (t & 1) * NC, tc::sw128_desc(ah), tc::sw128_desc(bh), IDESC, (t > 1 || kb > 0));
        }
        tc::mma_commit(FREE(s));
      }
      tc::mma_commit(DONE);  // arrives once every MMA issued above is complete
    }
    __syncwarp();
  } else {
    // ---------------- hi/lo conversion of the landed A box ----------------
    // this thread's 16-byte pieces tid + 128 i of the 16 KB tile: tile rows (tid >> 3) + 16 i
    // (the swizzle permutes pieces within a 128-byte row only)
    int rz[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = (tid >> 3) + 16 * i;
      const int64_t node = node0 + r / d;
      rz[i] = (r < rows_tile && node < p.N && jb.species) ? jb.species[node] : -1;
    }
    for (int t = 0; t < total; ++t) {
      const int s = t % NST, u = t / NST;
      if (!tc::mbar_wait_or_abort(FULL(s), u & 1, abort)) break;
      const int z = jb.species ? sZ[t / nchunks] : -1;
      const uint32_t st = base + s * S::STAGE;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t off = (uint32_t)(tid + 128 * i) * 16;
        float4 v;
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                     : "r"(st + off)
                     : "memory");
        if (rz[i] != z) v = make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 h = make_float4(tc::tf32_hi(v.x), tc::tf32_hi(v.y), tc::tf32_hi(v.z), tc::tf32_hi(v.w));
        const float4 l = make_float4(tc::tf32_hi(v.x - h.x), tc::tf32_hi(v.y - h.y), tc::tf32_hi(v.z - h.z),
                                     tc::tf32_hi(v.w - h.w));
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(st + off), "f"(h.x), "f"(h.y), "f"(h.z),
                     "f"(h.w)
                     : "memory");
        asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(st + S::A + off), "f"(l.x), "f"(l.y),
                     "f"(l.z), "f"(l.w)
                     : "memory");
      }
      tc::fence_proxy_async();  // the generic-proxy stores, visible to the tensor core
      tc::mbar_arrive(READY(s));
    }
  }
  __syncthreads();  // every role has left its loop; the abort flag is final
  const bool aborted = *abort != 0;
  bool done = true;
  if (warp < 4) done = tc::mbar_wait(DONE, 0);  // also before TMEM goes away after an abort
  if (aborted && warp == 4 && lane == 0) {
    // let the copies still in flight land before the shared memory goes away
    for (int t = (issued > NST ? issued - NST : 0); t < issued; ++t) tc::mbar_wait(FULL(t % NST), (t / NST) & 1);
  }
  if (warp < 4 && done && !aborted) {
    tc::fence_after_sync();
    // epilogue: warp w reads TMEM lanes 32w.. (tile rows), 32 columns at a time
    const int r = warp * 32 + lane;
    const int64_t node = node0 + r / d;
    float* const outp = jb.out ? jb.out : p.out;
    const int orow = jb.out ? jb.out_row : p.out_row;
    float* o = nullptr;
    if (r < rows_tile && node < p.N) o = outp + node * orow + jb.out_off + (r % d) * C + g * NC;
#pragma unroll 1
    for (int cb = 0; cb < NC / 32; ++cb) {
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + cb * 32;
      float4 y[8];
      if (o && jb.accumulate) {
        const float4* src = reinterpret_cast<const float4*>(o + cb * 32);
#pragma unroll
        for (int k = 0; k < 8; ++k) y[k] = src[k];
      }
      float v[32], x[32], w[32];
      tc::tmem_ld32(ta + 2 * NC, v);
      tc::tmem_ld32(ta, x);
      if (total > 1) tc::tmem_ld32(ta + NC, w);
      tc::tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] += x[k];
      if (total > 1) {
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] += w[k];
      }
      if (o) {
        float4* dst = reinterpret_cast<float4*>(o + cb * 32);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float4 e = make_float4(jb.alpha * v[4 * k], jb.alpha * v[4 * k + 1], jb.alpha * v[4 * k + 2],
                                 jb.alpha * v[4 * k + 3]);
          if (jb.accumulate) {
            e.x += y[k].x;
            e.y += y[k].y;
            e.z += y[k].z;
            e.w += y[k].w;
          }
          dst[k] = e;
        }
      }
    }
  }
  if (__syncthreads_or(aborted || !done) && tid == 0 && p.err_flag) atomicExch(p.err_flag, TC_ERR_TIMEOUT);
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, tl_tmem_cols<NC>());
  }
}

// operand image of the first N columns of a (K x ldb) row-major weight (per
// species z at w + z zstride): per 32-row K chunk, B[n][k] = W[k][n] as tf32
// hi then lo, each N rows x 128 bytes, 128B-swizzled
__global__ void k_tc_image(const float* __restrict__ w, int K, int ldb, int N, int Z, int64_t zstride,
                           float* __restrict__ img) {
  const int64_t total = (int64_t)Z * K * N;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int64_t r = i / N;
    const int k = (int)(r % K);
    const int z = (int)(r / K);
    const float v = w[z * zstride + (int64_t)k * ldb + n];
    const float hi = tc::tf32_hi(v);
    float* chunk = img + ((int64_t)z * (K / 32) + k / 32) * 2 * N * 32;
    const uint32_t off = tc::sw128_offset(n, k & 31, N) / 4;
    chunk[off] = hi;
    chunk[N * 32 + off] = tc::tf32_hi(v - hi);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult qr{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &qr) == cudaSuccess &&
        qr == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// nodes per row tile of a job whose rows have d entries per node
int tile_nodes(int d, int64_t N) { return (int)std::min<int64_t>(TL_ROWS / d, N); }

template <int NC>
int launch_tc(const LinTcParams& q, int grid, cudaStream_t s) {
  constexpr int BYTES = TlSmem<NC>::BYTES;
  static bool attr_set[64] = {};  // per device: the attribute call is slow on the host
  int dev = 0;
  MACE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !attr_set[dev]) {
    MACE_CUDA_TRY(cudaFuncSetAttribute(k_linear_tc<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES));
    if (dev < 64) attr_set[dev] = true;
  }
  k_linear_tc<NC><<<grid, TL_THREADS, BYTES, s>>>(q);
  MACE_LAUNCH_CHECK("linear_tc");
  return MACE_OK;
}

}  // namespace

int64_t tc_image_floats(int K, int N, int Z) { return (int64_t)Z * K * 2 * N; }

int launch_tc_image(const float* w, int K, int ldb, int N, int Z, int64_t zstride, float* img, cudaStream_t s) {
  if (K % 32 != 0 || N % 8 != 0) return fail(MACE_ERR_UNSUPPORTED, "tensor-core weight image shape");
  const int64_t total = (int64_t)Z * K * N;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  k_tc_image<<<blocks, 256, 0, s>>>(w, K, ldb, N, Z, zstride, img);
  MACE_LAUNCH_CHECK("tc_image");
  return MACE_OK;
}

bool linear_tc_supported(const LinParams& p) {
  if (p.C % 32 != 0 || p.C > 128 || p.C < 32) return false;
  if (p.in_row % 4 != 0 || p.N >= ((int64_t)1 << 31)) return false;
  if (!encode_tiled()) return false;
  int64_t rows = 0, maps = 0;
  for (int q = 0; q < p.n_jobs; ++q) {
    const LinJob& j = p.job[q];
    if (!j.tc || (reinterpret_cast<uintptr_t>(j.tc) & 15) != 0) return false;
    if (j.d < 1 || j.d > TL_ROWS) return false;
    for (int k = 0; k < j.n_k; ++k)
      if ((reinterpret_cast<uintptr_t>(p.in + j.k_off[k]) & 15) != 0) return false;
    maps += j.n_k;
    rows += p.N * j.d;
  }
  // below one full tile of rows the CUDA-core kernel's set-up is shorter
  return maps <= TL_MAX_MAPS && rows >= TL_ROWS;
}

int launch_linear_tc(const LinParams& p, cudaStream_t s) {
  EncodeTiledFn encode = encode_tiled();
  if (!encode) return fail(MACE_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled is not available");
  LinTcParams q{};
  q.p = p;
  int items = 0, nmaps = 0;
  for (int j = 0; j < p.n_jobs; ++j) {
    const LinJob& jb = p.job[j];
    const int tn = tile_nodes(jb.d, p.N);
    q.tn[j] = tn;
    q.tile_start[j] = items;
    q.map_base[j] = nmaps;
    items += (int)((p.N + tn - 1) / tn);
    for (int k = 0; k < jb.n_k; ++k) {
      if (nmaps >= TL_MAX_MAPS) return fail(MACE_ERR_UNSUPPORTED, "tensor-core linear: too many input slots");
      const cuuint64_t dims[3] = {(cuuint64_t)p.C, (cuuint64_t)jb.d, (cuuint64_t)p.N};
      const cuuint64_t strides[2] = {(cuuint64_t)p.C * 4, (cuuint64_t)p.in_row * 4};
      const cuuint32_t box[3] = {32, (cuuint32_t)jb.d, (cuuint32_t)tn};
      const cuuint32_t estr[3] = {1, 1, 1};
      const CUresult r = encode(&q.map[nmaps], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                                const_cast<float*>(p.in + jb.k_off[k]), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      if (r != CUDA_SUCCESS)
        return fail(MACE_ERR_CUDA, "cuTensorMapEncodeTiled failed for a node-linear input (code " +
                                       std::to_string((int)r) + ")");
      ++nmaps;
    }
  }
  q.tile_start[p.n_jobs] = items;
  if (items == 0) return MACE_OK;
  // column groups: a CTA's chunk loop is latency-bound, so the narrowest NC
  // whose CTAs still run in one wave (one CTA per SM); full width otherwise
  static int sm_count[64] = {};
  int dev = 0;
  MACE_CUDA_TRY(cudaGetDevice(&dev));
  int sms = dev < 64 ? sm_count[dev] : 0;
  if (sms == 0) {
    MACE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (dev < 64) sm_count[dev] = sms;
  }
  int nc = p.C;
  for (int cand : {p.C / 4, p.C / 3, p.C / 2}) {
    if (cand < 32 || cand % 32 != 0 || p.C % cand != 0) continue;
    if ((int64_t)items * (p.C / cand) <= sms) {
      nc = cand;
      break;
    }
  }
  q.cs = p.C / nc;
  const int grid = items * q.cs;
  switch (nc) {
    case 32: return launch_tc<32>(q, grid, s);
    case 64: return launch_tc<64>(q, grid, s);
    case 96: return launch_tc<96>(q, grid, s);
    case 128: return launch_tc<128>(q, grid, s);
    default: return fail(MACE_ERR_UNSUPPORTED, "tensor-core linear channel count");
  }
}

}  // namespace mace
