// Node linears (o3.Linear, the skip_tp's species-indexed channel mixing and
// their transposes) on the 5th-generation tensor cores.
//
// A job maps rows (node, m) of its concat-K input slots to one output slot:
//   out[n, out_off + m C + o] (+)= alpha * sum_k in[n, k_off[k/C] + m C + k%C] W[k][o].
// One CTA computes a 128-row x C tile of one job in TMEM (128 lanes x C fp32
// columns per accumulator) over 32-wide K chunks t:
//   D_small += A_lo B_hi + A_hi B_lo,   D_big[t & 1] += A_hi B_hi
// (kind::tf32, 4 K-steps of 8) with A the 128 x 32 input chunk and B the
// weight chunk (C rows x 32, the transpose of W's 32 rows); hi = x rounded to
// tf32, lo = (x - hi) rounded to tf32 (the 3xTF32 split), and the epilogue
// adds the three accumulators in fp32.  The tensor core truncates when it
// accumulates, and the error grows with the number of accumulation steps into
// one accumulator: the small terms in their own accumulator and two
// alternating big ones keep it near fp32 rounding.  The weights never change, so their operand
// images (tf32 hi and lo, 128B-swizzled K-major) are made once per context
// (k_tc_image); a chunk's image is one contiguous bulk copy.  The input chunk
// is read with coalesced 16-byte loads (8 threads per 128-byte row segment),
// split into hi/lo in registers and stored straight into the swizzled
// operand tiles.  Three stages: the loads of chunk t+1 are in flight while
// chunk t is stored and its MMAs run.
//
// Species-indexed jobs (the skip connection) run one pass per distinct
// species in the tile, with the rows of other species zeroed in A and that
// species' weight image in B.
//
// Every mbarrier wait is bounded (about 2 s).  A wait that gives up makes the
// whole CTA leave the K loop (agreed through __syncthreads_or), wait (bounded)
// for its MMAs, record TC_ERR_TIMEOUT in the error flag, free its TMEM and
// return.
#include "common.cuh"
#include "tc.cuh"

namespace mace {

namespace {

constexpr int TL_STAGES = 3;
constexpr int TL_ROWS = 128;
constexpr int TL_THREADS = 192;  // warps 0-3: A chunks + epilogue; 4: weight copies; 5: MMAs

template <int NC>
__host__ __device__ constexpr uint32_t tl_tmem_cols() {
  return 3 * NC <= 128 ? 128 : (3 * NC <= 256 ? 256 : 512);
}

template <int NC>
struct TlSmem {
  static constexpr int A = TL_ROWS * 128;  // one 128-row x 32 fp32 operand tile
  static constexpr int B = NC * 128;       // one NC-row x 32 operand tile
  static constexpr int STAGE = 2 * A + 2 * B;  // A hi, A lo, B hi, B lo
  static constexpr int BYTES = TL_STAGES * STAGE + 1024;  // + alignment slack
};

template <int NC>
__global__ void __launch_bounds__(TL_THREADS, 1) k_linear_tc(const __grid_constant__ LinParams p) {
  using S = TlSmem<NC>;
  extern __shared__ uint8_t smem_raw[];
  // full[s] (weight copy landed), ready[s] (A chunk stored), free[s] (MMAs done), done
  __shared__ __align__(8) uint64_t bars[3 * TL_STAGES + 1];
  __shared__ uint32_t tslot;
  __shared__ int abort_flag;
  __shared__ uint32_t zmask[8];
  __shared__ int sZ[TL_ROWS + 1];
  const LinJob& jb = p.job[blockIdx.y];
  const int C = p.C;
  const int rows = (int)(p.N * jb.d);
  const int r0 = blockIdx.x * TL_ROWS;
  if (r0 >= rows) return;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t base = (tc::smem_u32(smem_raw) + 1023u) & ~1023u;
  auto FULL = [&](int s) { return tc::smem_u32(&bars[s]); };
  auto READY = [&](int s) { return tc::smem_u32(&bars[TL_STAGES + s]); };
  auto FREE = [&](int s) { return tc::smem_u32(&bars[2 * TL_STAGES + s]); };
  const uint32_t DONE = tc::smem_u32(&bars[3 * TL_STAGES]);
  volatile int* abort = &abort_flag;

  if (warp == 0) {
    tc::tmem_alloc(tc::smem_u32(&tslot), tl_tmem_cols<NC>());
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < TL_STAGES; ++s) {
      tc::mbar_init(FULL(s), 1);
      tc::mbar_init(READY(s), 128);
      tc::mbar_init(FREE(s), 1);
    }
    tc::mbar_init(DONE, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
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
    if (tid < TL_ROWS && r0 + tid < rows) {
      const int z = jb.species[(r0 + tid) / jb.d];
      if (z < 256)
        atomicOr(&zmask[z >> 5], 1u << (z & 31));
      else
        wide = true;
    }
    if (__syncthreads_or(wide)) {  // species index beyond the mask: serial scan
      if (tid == 0) {
        int nd = 0;
        for (int q = 0; q < TL_ROWS && r0 + q < rows; ++q) {
          const int z = jb.species[(r0 + q) / jb.d];
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
  const int nck = C / 32;
  const int nchunks = jb.n_k * nck;
  const int total = n_pass * nchunks;
  const int64_t zimg = (int64_t)nchunks * 2 * NC * 32;  // floats of one species' image
  constexpr uint32_t IDESC = tc::idesc_tf32(TL_ROWS, NC);
  int issued = 0;  // weight copies issued (warp 4, lane 0)

  if (warp == 4) {
    // ---------------- weight copies ----------------
    if (lane == 0) {
      for (int t = 0; t < total; ++t) {
        const int s = t % TL_STAGES, u = t / TL_STAGES;
        if (t >= TL_STAGES && !tc::mbar_wait_or_abort(FREE(s), (u - 1) & 1, abort)) break;
        const int pass = t / nchunks, tt = t - pass * nchunks;
        const int z = jb.species ? sZ[pass] : 0;
        tc::mbar_expect_tx(FULL(s), 2 * S::B);
        tc::bulk_g2s(base + s * S::STAGE + 2 * S::A, jb.tc + z * zimg + (int64_t)tt * 2 * NC * 32, 2 * S::B,
                     FULL(s));
        ++issued;
      }
    }
    __syncwarp();
  } else if (warp == 5) {
    // ---------------- MMAs ----------------
    if (lane == 0) {
      for (int t = 0; t < total; ++t) {
        const int s = t % TL_STAGES, u = t / TL_STAGES;
        if (!tc::mbar_wait_or_abort(FULL(s), u & 1, abort)) break;
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
    // ---------------- A chunks: coalesced loads, tf32 split, swizzled stores ----------------
    // this thread's 16-byte column j4 of rows (tid >> 3) + 16 i
    const int j4 = tid & 7;
    const float* rp[8];
    int rz[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = r0 + (tid >> 3) + 16 * i;
      rp[i] = nullptr;
      rz[i] = -1;
      if (row < rows) {
        const int node = row / jb.d, m = row - node * jb.d;
        rp[i] = p.in + (int64_t)node * p.in_row + m * C + 4 * j4;
        rz[i] = jb.species ? jb.species[node] : 0;
      }
    }
    auto load = [&](int t, float4(&ra)[8]) {
      const int pass = t / nchunks, tt = t - pass * nchunks;
      const int ks = tt / nck, kc = tt - ks * nck;
      const int z = jb.species ? sZ[pass] : 0;
      const int off = jb.k_off[ks] + 32 * kc;
#pragma unroll
      for (int i = 0; i < 8; ++i)
        ra[i] = (rp[i] && rz[i] == z) ? __ldg(reinterpret_cast<const float4*>(rp[i] + off))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto store = [&](int t, float4(&ra)[8]) -> bool {
      const int s = t % TL_STAGES, u = t / TL_STAGES;
      if (t >= TL_STAGES && !tc::mbar_wait_or_abort(FREE(s), (u - 1) & 1, abort)) return false;
      const uint32_t st = base + s * S::STAGE;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = (tid >> 3) + 16 * i;
        const uint32_t off = r * 128 + ((j4 ^ (r & 7)) << 4);
        const float4 v = ra[i];
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
      if (t + 2 < total) load(t + 2, ra);
      tc::fence_proxy_async();  // the generic-proxy stores, visible to the tensor core
      tc::mbar_arrive(READY(s));
      return true;
    };
    float4 ra0[8], ra1[8];
    load(0, ra0);
    if (total > 1) load(1, ra1);
    for (int t = 0; t < total; t += 2) {
      if (!store(t, ra0)) break;
      if (t + 1 < total && !store(t + 1, ra1)) break;
    }
  }
  __syncthreads();  // every role has left its loop; the abort flag is final
  const bool aborted = *abort != 0;
  bool done = true;
  if (warp < 4) done = tc::mbar_wait(DONE, 0);  // also before TMEM goes away after an abort
  if (aborted && warp == 4 && lane == 0) {
    // let the weight copies still in flight land before the shared memory goes away
    for (int t = (issued > TL_STAGES ? issued - TL_STAGES : 0); t < issued; ++t)
      tc::mbar_wait(FULL(t % TL_STAGES), (t / TL_STAGES) & 1);
  }
  if (warp < 4 && done && !aborted) {
    tc::fence_after_sync();
    // epilogue: warp w reads TMEM lanes 32w.. (tile rows), 32 columns at a time
    const int row = r0 + warp * 32 + lane;
    float* const outp = jb.out ? jb.out : p.out;
    const int orow = jb.out ? jb.out_row : p.out_row;
    float* o = nullptr;
    if (row < rows) {
      const int node = row / jb.d, m = row - node * jb.d;
      o = outp + (int64_t)node * orow + jb.out_off + m * C;
    }
#pragma unroll 1
    for (int cb = 0; cb < NC / 32; ++cb) {
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + cb * 32;
      float v[32], x[32];
      tc::tmem_ld32(ta + 2 * NC, v);
      tc::tmem_ld32(ta, x);
      tc::tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 32; ++q) v[q] += x[q];
      if (total > 1) {
        tc::tmem_ld32(ta + NC, x);
        tc::tmem_wait_ld();
#pragma unroll
        for (int q = 0; q < 32; ++q) v[q] += x[q];
      }
      if (o) {
        float4* dst = reinterpret_cast<float4*>(o + cb * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 w = make_float4(jb.alpha * v[4 * q], jb.alpha * v[4 * q + 1], jb.alpha * v[4 * q + 2],
                                 jb.alpha * v[4 * q + 3]);
          if (jb.accumulate) {
            const float4 y = dst[q];
            w.x += y.x;
            w.y += y.y;
            w.z += y.z;
            w.w += y.w;
          }
          dst[q] = w;
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

template <int NC>
int launch_tc(const LinParams& p, int max_rows, cudaStream_t s) {
  constexpr int BYTES = TlSmem<NC>::BYTES;
  static bool attr_set[64] = {};  // per device: the attribute call is slow on the host
  int dev = 0;
  MACE_CUDA_TRY(cudaGetDevice(&dev));
  if (dev >= 64 || !attr_set[dev]) {
    MACE_CUDA_TRY(cudaFuncSetAttribute(k_linear_tc<NC>, cudaFuncAttributeMaxDynamicSharedMemorySize, BYTES));
    if (dev < 64) attr_set[dev] = true;
  }
  dim3 grid((max_rows + TL_ROWS - 1) / TL_ROWS, p.n_jobs);
  k_linear_tc<NC><<<grid, TL_THREADS, BYTES, s>>>(p);
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
  if (p.in_row % 4 != 0) return false;
  int64_t work = 0;  // rows x K over the jobs
  bool all_species = true;
  for (int q = 0; q < p.n_jobs; ++q) {
    const LinJob& j = p.job[q];
    if (!j.tc) return false;
    if ((reinterpret_cast<uintptr_t>(j.tc) & 15) != 0) return false;
    for (int k = 0; k < j.n_k; ++k)
      if (j.k_off[k] % 4 != 0) return false;
    work += p.N * j.d * (int64_t)j.n_k * p.C;
    all_species = all_species && j.species != nullptr;
  }
  // A 128-row tile walks its K chunks one after another, so a launch with few
  // tiles is latency-bound; there the CUDA-core kernel's 32-row tiles spread
  // the same work over more SMs and finish first (measured on B200 at 1000
  // nodes: break-even near 4000 rows of K = 128, twice that for the
  // species-indexed skip).
  return work >= (all_species ? 2 : 1) * 4000LL * 128;
}

int launch_linear_tc(const LinParams& p, cudaStream_t s) {
  int max_rows = 0;
  for (int q = 0; q < p.n_jobs; ++q) max_rows = std::max(max_rows, (int)(p.N * p.job[q].d));
  if (max_rows == 0) return MACE_OK;
  switch (p.C) {
    case 32: return launch_tc<32>(p, max_rows, s);
    case 64: return launch_tc<64>(p, max_rows, s);
    case 96: return launch_tc<96>(p, max_rows, s);
    case 128: return launch_tc<128>(p, max_rows, s);
    default: return fail(MACE_ERR_UNSUPPORTED, "tensor-core linear channel count");
  }
}

}  // namespace mace
