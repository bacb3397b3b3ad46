// Radial MLP on the 5th-generation tensor cores (sm_100a tcgen05, kind::tf32
// with a 3-term hi/lo split for fp32-level accuracy; see tc.cuh).
//
// One CTA owns a tile of 128 edges (TMEM lane t = edge t of the tile) and runs
// nine warps: eight epilogue warps (quadrant q = warp & 3 owns TMEM lanes /
// edges 32q..32q+31, group g = warp >> 2 owns half of the columns) and a
// control warp whose lane 0 issues every bulk copy and every tcgen05.mma.  The
// warps hand work to one another through mbarriers only.  The activation-side
// operand A of every MMA lives in TMEM (written with tcgen05.st, read by the
// MMA), so shared memory only holds weight images, copy stages and output
// staging; two CTAs per SM (256 of the SM's 512 TMEM columns each, 96
// registers per thread).
//
// Forward:
//   layer 0 (radial features -> 64) on the CUDA cores; every 64 x 64 hidden
//   layer as 8 K-blocks x 3 MMAs (M = 128, N = 64, K = 8) with a pre-split,
//   pre-swizzled weight image (B); the last layer in 64-column chunks (MMA
//   N = 64: a tcgen05.mma costs about the same issue time at N = 32 as at
//   N = 128, so wide chunks halve the instruction count per output column)
//   with two B stages (the next chunk's image copied while this one
//   multiplies) and two TMEM accumulators; both epilogue groups drain every
//   chunk, group g its 32-column half, each warp moving its 32 rows of the
//   half from TMEM through a 4 KB staging slice to HBM with one bulk store:
//   the output is in the 128-edge tile layout (common.cuh), whose 32-column
//   chunk rows are exactly a staging slice.
// Backward:
//   dH = dW (128 x W) . W_last^T in 32-wide K chunks through three copy
//   stages: the control warp bulk-copies a 16 KB dW chunk (already in operand
//   layout) and the matching 16 KB weight image (hi rows then lo rows), the
//   epilogue warps split the chunk into tf32 hi (in place) and lo (TMEM), and
//   the control warp issues per K-block one N = 128 MMA of A_hi against the
//   stacked hi|lo weight rows (the large term and one small term side by
//   side) and one N = 64 MMA of A_lo against the hi rows; then every hidden
//   layer dH <- (dH * SiLU'(a)) . W_j^T on the tensor cores, and dL/db on the
//   CUDA cores.
//
// Every mbarrier wait is bounded (about 2 s).  A wait that gives up raises a
// CTA-wide abort flag that ends every other wait, the kernel records
// MLP_TC_TIMEOUT in the error flag, frees its TMEM and returns.
#include "common.cuh"
#include "tc.cuh"

namespace mace {

namespace {

constexpr int TM = 128;           // edges per tile (MMA M)
constexpr int H = 64;             // hidden width
constexpr int FC = 64;            // output columns per forward chunk (MMA N)
constexpr int KC = 32;            // backward K chunk (one 128-byte panel)
constexpr int NBUF = 2;           // forward TMEM chunk buffers of FC columns
constexpr int MLP_TC_TIMEOUT = TC_ERR_TIMEOUT;
constexpr int MLP_TC_ALIGN = TC_ERR_ALIGN;
constexpr int IMG = 2 * H * H;    // floats of one 64 x 64 hi/lo image
constexpr int CIMG = 2 * FC * H;    // floats of one forward chunk image (64 x 64, hi/lo)
constexpr int BIMG = 2 * H * KC;    // floats of one backward chunk image (64 x 32, hi/lo)
static_assert(WT_CHUNK * 4 == TM * 128, "a radial-weight chunk is one 128 x 128-byte operand panel");

// the (NB, 64) layer-0 weights into shared memory by the 128 epilogue threads
template <int NB>
__device__ __forceinline__ void load_w0(const MlpParams& p, float* sW0, int t) {
  for (int q = t; q < NB * H / 4; q += TM)
    reinterpret_cast<float4*>(sW0)[q] = __ldg(reinterpret_cast<const float4*>(p.w[0]) + q);
  tc::named_sync(1, TM);
}

// layer 0 on the CUDA cores: y = b[e] . W0 (shared-memory broadcast reads)
template <int NB>
__device__ __forceinline__ void layer0(const MlpParams& p, const float* sW0, int64_t e, bool valid, float* y) {
  float x[NB];
#pragma unroll
  for (int i = 0; i < NB; ++i) x[i] = valid ? __ldg(p.b + e * NB + i) : 0.f;
#pragma unroll
  for (int o = 0; o < H; ++o) y[o] = 0.f;
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const float4* w4 = reinterpret_cast<const float4*>(sW0 + i * H);
#pragma unroll
    for (int q = 0; q < H / 4; ++q) {
      const float4 w = w4[q];
      y[4 * q + 0] = fmaf(x[i], w.x, y[4 * q + 0]);
      y[4 * q + 1] = fmaf(x[i], w.y, y[4 * q + 1]);
      y[4 * q + 2] = fmaf(x[i], w.z, y[4 * q + 2]);
      y[4 * q + 3] = fmaf(x[i], w.w, y[4 * q + 3]);
    }
  }
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
constexpr int F_NEPI = 8;                 // epilogue warps: quadrant q = warp & 3, group g = warp >> 2
constexpr int F_NTHR = 32 * (F_NEPI + 1); // + control warp
constexpr int F_TMEM = 256;               // [0, 128) accumulators, [128, 192) A hi, [192, 256) A lo
constexpr uint32_t F_AHI = 128, F_ALO = 192;
constexpr uint32_t F_HSMALL = 64;  // small-term accumulator of the hidden layers (chunk buffer 1 meanwhile free)

constexpr int F_NBS = 2;  // forward chunk-image stages
struct FwdSmem {
  // 64 KB: two 64-row chunk images; the 64 x 64 hidden image uses the first 32 KB
  static constexpr int B = 0;
  static constexpr int STG = F_NBS * CIMG * 4;  // 8 warps x 4 KB output staging; holds the layer-0 weights first
  static constexpr int BARS = STG + F_NEPI * 4096;
  static constexpr int TOTAL = BARS + 256;
  // request enough to keep two CTAs per SM (each holds 256 of the SM's 512 TMEM columns)
  static constexpr int REQUEST = 100 * 1024;
  static constexpr int TL = 0, A = 1, ACC = 2, BST = 3, FULL = BST + F_NBS, FREE = FULL + NBUF,
                       NBARS = FREE + NBUF;
};
static_assert(FwdSmem::TOTAL <= FwdSmem::REQUEST, "forward shared memory");

// The tensor core does not round to nearest when it adds into an fp32
// accumulator: every accumulation step can lose up to one unit in the last
// place of the running sum, always in the same direction.  The two small
// cross terms of the 3xTF32 product (hi.lo, lo.hi) therefore never go into
// the running sum of the large hi.hi term: they get their own accumulator
// (whose magnitude is 2^-11 of the large one, so its steps are harmless), or,
// where no TMEM is free, they are issued first while the running sum is
// still small; the two sums are added in fp32 on the CUDA cores.

// D_big (+)= A_hi . B_hi^T and D_small (+)= A_hi . B_lo^T + A_lo . B_hi^T over K = 64
// (D 128 x N, A in TMEM 128 x 64, B N x 64), issued by one thread
template <int N>
__device__ __forceinline__ void mma_k64_split(uint32_t d_big, uint32_t d_small, uint32_t a_hi, uint32_t a_lo,
                                              uint32_t b_hi, uint32_t b_lo) {
  constexpr uint32_t IDESC = tc::idesc_tf32(TM, N);
#pragma unroll
  for (int kb = 0; kb < H / 8; ++kb) {
    const uint32_t ob = (kb >> 2) * (N * 128) + (kb & 3) * 32;
    tc::mma_tf32_ta(d_small, a_hi + kb * 8, tc::sw128_desc(b_lo + ob), IDESC, kb > 0);
    tc::mma_tf32_ta(d_small, a_lo + kb * 8, tc::sw128_desc(b_hi + ob), IDESC, 1);
  }
#pragma unroll
  for (int kb = 0; kb < H / 8; ++kb) {
    const uint32_t ob = (kb >> 2) * (N * 128) + (kb & 3) * 32;
    tc::mma_tf32_ta(d_big, a_hi + kb * 8, tc::sw128_desc(b_hi + ob), IDESC, kb > 0);
  }
}

// D (128 x N) = A . B^T in one accumulator, the small cross terms first
template <int N>
__device__ __forceinline__ void mma_k64_ta(uint32_t tmem_d, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi,
                                           uint32_t b_lo) {
  constexpr uint32_t IDESC = tc::idesc_tf32(TM, N);
#pragma unroll
  for (int kb = 0; kb < H / 8; ++kb) {
    const uint32_t ob = (kb >> 2) * (N * 128) + (kb & 3) * 32;
    tc::mma_tf32_ta(tmem_d, a_hi + kb * 8, tc::sw128_desc(b_lo + ob), IDESC, kb > 0);
    tc::mma_tf32_ta(tmem_d, a_lo + kb * 8, tc::sw128_desc(b_hi + ob), IDESC, 1);
  }
#pragma unroll
  for (int kb = 0; kb < H / 8; ++kb) {
    const uint32_t ob = (kb >> 2) * (N * 128) + (kb & 3) * 32;
    tc::mma_tf32_ta(tmem_d, a_hi + kb * 8, tc::sw128_desc(b_hi + ob), IDESC, 1);
  }
}

// One CTA per 128-edge tile, 8 epilogue warps + 1 control warp, two CTAs per SM.
// The activation operand A lives in TMEM (written with tcgen05.st), so shared
// memory only holds the weight images (two 64-column chunk stages, each
// refilled as soon as the MMA that read it completes) and one 4 KB output
// staging slice per epilogue warp, whose bulk store drains while the warp's
// group waits for its next chunk.  Each 64-column chunk accumulates into one
// of two TMEM buffers; epilogue group g drains its 32-column half 2c + g.
template <int NB>
__global__ void __maxnreg__(96) k_mlp_fwd_tc(MlpParams p) {
  extern __shared__ __align__(1024) unsigned char sm[];
  using S = FwdSmem;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if ((tc::smem_u32(sm) & 1023u) != 0) {
    if (t == 0) atomicExch(p.err_flag, MLP_TC_ALIGN);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + S::BARS + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::BARS + 136);
  auto BAR = [&](int i) { return tc::smem_u32(&bars[i]); };
  const int nh = p.n_layers - 1;
  const int wout = p.widths[p.n_layers];
  const int nch = wt_nchunk(wout);  // 32-column chunks of the output layout
  const int nfc = (nch + 1) / 2;    // 64-column MMA chunks
  const uint32_t b_base = tc::smem_u32(sm + S::B);

  if (warp == F_NEPI) {
    tc::tmem_alloc(tc::smem_u32(tslot), F_TMEM);
    tc::tmem_relinquish();
  }
  if (t == 0) {
    for (int i = 0; i < S::NBARS; ++i) {
      int count = 1;
      if (i == S::A) count = F_NEPI;
      if (i >= S::FREE && i < S::FREE + NBUF) count = F_NEPI;  // both groups drain every buffer
      tc::mbar_init(BAR(i), count);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  bool ok = true;

  if (warp == F_NEPI) {
    // ---------------- control warp: copies and MMAs from lane 0 ----------------
    if (lane == 0) {
      auto wait = [&](int i, uint32_t par) {
        ok = ok && tc::mbar_wait_or_abort(BAR(i), par, abort_flag);
        return ok;
      };
      auto copy_trunk = [&](int j) {
        tc::mbar_expect_tx(BAR(S::TL), IMG * 4);
        tc::bulk_g2s(b_base, p.tc_trunk + (int64_t)j * IMG, IMG * 4, BAR(S::TL));
      };
      auto copy_chunk = [&](int c) {
        const int s = c % F_NBS;
        tc::mbar_expect_tx(BAR(S::BST + s), CIMG * 4);
        tc::bulk_g2s(b_base + s * CIMG * 4, p.tc_img + (int64_t)c * CIMG, CIMG * 4, BAR(S::BST + s));
      };
      const uint32_t a_hi = tmem + F_AHI, a_lo = tmem + F_ALO;
      uint32_t pa = 0;
      // chunk image 1 does not overlap the hidden-layer image: fetch it now
      if (nfc > 1) copy_chunk(1);
      if (nh >= 2) copy_trunk(0);
      for (int j = 1; j < nh; ++j) {  // hidden layer j reads A = SiLU(layer j-1)
        if (!wait(S::TL, (j - 1) & 1) || !wait(S::A, pa)) break;
        pa ^= 1;
        tc::fence_after_sync();
        mma_k64_split<H>(tmem, tmem + F_HSMALL, a_hi, a_lo, b_base, b_base + IMG * 2);
        tc::mma_commit(BAR(S::ACC));
        if (!wait(S::ACC, (j - 1) & 1)) break;  // B is free again
        if (j + 1 < nh) copy_trunk(j);
      }
      if (ok) copy_chunk(0);  // the hidden-layer image is no longer read
      if (ok && wait(S::A, pa)) {  // A = SiLU(last hidden layer)
        for (int c = 0; c < nfc; ++c) {
          const int s = c % F_NBS, buf = c % NBUF;
          if (!wait(S::BST + s, (c / F_NBS) & 1)) break;
          if (c >= NBUF && !wait(S::FREE + buf, ((c / NBUF) - 1) & 1)) break;
          tc::fence_after_sync();
          const uint32_t bs = b_base + s * CIMG * 4;
          mma_k64_ta<FC>(tmem + buf * FC, a_hi, a_lo, bs, bs + CIMG * 2);
          tc::mma_commit(BAR(S::FULL + buf));
          // stage (c - 1) % F_NBS is free once MMA(c - 1) is done: chunk c + F_NBS - 1 goes there
          if (c >= 1 && c + F_NBS - 1 < nfc) {
            if (!wait(S::FULL + (c - 1) % NBUF, ((c - 1) / NBUF) & 1)) break;
            copy_chunk(c + F_NBS - 1);
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps: row = TMEM lane, columns split by group ----------------
    const int q = warp & 3, g = warp >> 2;
    const int row = q * 32 + lane;
    const int64_t e = (int64_t)blockIdx.x * TM + row;
    const bool valid = e < p.E;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    auto wwait = [&](int i, uint32_t par) {
      const bool r = ok && tc::mbar_wait_or_abort(BAR(i), par, abort_flag);
      ok = __all_sync(0xffffffffu, r);
      return ok;
    };
    // layer 0 on the CUDA cores for this group's 32 hidden columns
    float* sW0 = reinterpret_cast<float*>(sm + S::STG);
    for (int i = t; i < NB * H / 4; i += 32 * F_NEPI)
      reinterpret_cast<float4*>(sW0)[i] = __ldg(reinterpret_cast<const float4*>(p.w[0]) + i);
    tc::named_sync(1, 32 * F_NEPI);
    float y[32];
    {
      float x[NB];
#pragma unroll
      for (int i = 0; i < NB; ++i) x[i] = valid ? __ldg(p.b + e * NB + i) : 0.f;
#pragma unroll
      for (int o = 0; o < 32; ++o) y[o] = 0.f;
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const float4* w4 = reinterpret_cast<const float4*>(sW0 + i * H + 32 * g);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 w = w4[k];
          y[4 * k + 0] = fmaf(x[i], w.x, y[4 * k + 0]);
          y[4 * k + 1] = fmaf(x[i], w.y, y[4 * k + 1]);
          y[4 * k + 2] = fmaf(x[i], w.z, y[4 * k + 2]);
          y[4 * k + 3] = fmaf(x[i], w.w, y[4 * k + 3]);
        }
      }
    }
    uint32_t pacc = 0;
    for (int j = 0; j < nh; ++j) {
      if (valid) {
        float4* act = reinterpret_cast<float4*>(p.act + e * (int64_t)(nh * H) + j * H + 32 * g);
#pragma unroll
        for (int k = 0; k < 8; ++k) act[k] = make_float4(y[4 * k], y[4 * k + 1], y[4 * k + 2], y[4 * k + 3]);
      }
#pragma unroll
      for (int o = 0; o < 32; ++o) y[o] = valid ? silu_f(y[o]) : 0.f;
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {  // 16 columns at a time keeps the temporaries small
        float part[16];
#pragma unroll
        for (int o = 0; o < 16; ++o) part[o] = tc::tf32_hi(y[16 * hf + o]);
        tc::tmem_st16(tmem + lane_base + F_AHI + 32 * g + 16 * hf, part);
#pragma unroll
        for (int o = 0; o < 16; ++o) part[o] = y[16 * hf + o] - tc::tf32_hi(y[16 * hf + o]);
        tc::tmem_st16(tmem + lane_base + F_ALO + 32 * g + 16 * hf, part);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(BAR(S::A));
      if (j + 1 < nh) {
        if (!wwait(S::ACC, pacc)) break;
        pacc ^= 1;
        tc::fence_after_sync();
        tc::tmem_ld32(tmem + lane_base + 32 * g, y);
        tc::tmem_wait_ld();
        tc::tmem_ld16_add(tmem + lane_base + F_HSMALL + 32 * g, y);
        tc::tmem_ld16_add(tmem + lane_base + F_HSMALL + 32 * g + 16, y + 16);
      }
    }
    // output chunk 2c + g (columns 32g.. of MMA chunk c): TMEM -> registers -> staging -> bulk store
    float* dst = p.out + (int64_t)blockIdx.x * nch * WT_CHUNK + q * 32 * 32;
    for (int c = 0; c < nfc && ok; ++c) {
      const int buf = c % NBUF;
      if (!wwait(S::FULL + buf, (c / NBUF) & 1)) break;
      tc::fence_after_sync();
      float v[32];
      tc::tmem_ld32(tmem + lane_base + buf * FC + 32 * g, v);
      tc::tmem_wait_ld();
      tc::fence_before_sync();
      __syncwarp();
      unsigned char* stg = sm + S::STG + warp * 4096;
      if (lane == 0) {
        tc::mbar_arrive(BAR(S::FREE + buf));
        tc::bulk_wait_read_all();  // this warp's previous store has read its staging buffer
      }
      __syncwarp();
#pragma unroll
      for (int u = 0; u < 8; ++u)
        *reinterpret_cast<float4*>(stg + lane * 128 + ((u ^ (lane & 7)) << 4)) =
            make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
      tc::fence_proxy_async();
      __syncwarp();
      if (lane == 0 && 2 * c + g < nch) {  // an odd chunk count leaves the last half unwritten
        tc::bulk_s2g(dst + (int64_t)(2 * c + g) * WT_CHUNK, tc::smem_u32(stg), 4096);
        tc::bulk_commit();
      }
    }
    if (lane == 0) tc::bulk_wait_all();
    __syncwarp();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (!ok) atomicExch(p.err_flag, MLP_TC_TIMEOUT);
  if (warp == F_NEPI) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, F_TMEM);
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------
constexpr int B_NST = 3;  // copy stages of (dW chunk, weight chunk image)
constexpr int B_GROUP = 2;  // K chunks per dH partial sum (drained to fp32 registers, see below)
// The dW chunk's tf32 hi part is the MMA's A operand straight from shared
// memory (the epilogue rounds the bulk-copied chunk in place; it is already in
// the 128B-swizzled K-major operand layout) and only its lo part goes to TMEM.
// TMEM: the dH partial sum of the current chunk group, hi.hi at [0, 64) and
// the two small terms at [64, 128) (one N = 128 MMA writes both halves);
// stage s's lo part at 128 + 32 s; after the K loop the hidden layers' A
// (128 x 64) at [128, 192) hi, [192, 256) lo, their hi.hi accumulator at
// [0, 64) and small-term accumulator at [64, 128)
constexpr uint32_t B_ALO = 128, B_TAHI = 128, B_TALO = 192, B_SMALL = 64;

struct BwdSmem {
  // stage s at s * STAGE: the dW chunk (16 KB, bulk-copied in the 128-edge tile
  // layout, which is the operand layout) and the weight chunk image (16 KB);
  // after the K loop the hidden layers' weight image uses [0, 32K)
  static constexpr int STAGE = 32768;
  static constexpr int W0 = B_NST * STAGE;       // layer-0 weights (NB, 64), <= 4 KB
  static constexpr int DB = STAGE;               // at the end: 128 rows x 2 groups x 16 partial dL/db (stage 1)
  static constexpr int BARS = W0 + 4096;
  static constexpr int TOTAL = BARS + 256;
  static constexpr int REQUEST = 112 * 1024;     // two CTAs per SM (256 TMEM columns each)
  static constexpr int LD = 0, SPLIT = 3, MMA = 6, TL = 9, A = 10, ACC = 11, DRAIN = 12, NBARS = 14;
};
static_assert(BwdSmem::TOTAL <= BwdSmem::REQUEST, "backward shared memory");

// dH = dW . W_last^T in 32-wide K chunks: the control warp bulk-copies each
// dW chunk and its weight image into one of three stages; the epilogue warps
// (quadrant q = rows, group g = 16 of the chunk's 32 columns) split the chunk
// into tf32 hi/lo straight into TMEM (tcgen05.st) for the MMAs, which read A
// from TMEM; the hidden layers follow as in the forward, and dL/db on the
// CUDA cores with the two column halves summed through shared memory.
template <int NB>
__global__ void __maxnreg__(96) k_mlp_bwd_tc(MlpParams p) {
  extern __shared__ __align__(1024) unsigned char sm[];
  using S = BwdSmem;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if ((tc::smem_u32(sm) & 1023u) != 0) {
    if (t == 0) atomicExch(p.err_flag, MLP_TC_ALIGN);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + S::BARS);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + S::BARS + 128);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(sm + S::BARS + 136);
  auto BAR = [&](int i) { return tc::smem_u32(&bars[i]); };
  const int nh = p.n_layers - 1;
  const int wout = p.widths[p.n_layers];
  const int nch = wt_nchunk(wout);
  const int last = nch - 1;
  const uint32_t base = tc::smem_u32(sm);

  if (warp == F_NEPI) {
    tc::tmem_alloc(tc::smem_u32(tslot), F_TMEM);
    tc::tmem_relinquish();
  }
  if (t == 0) {
    for (int i = 0; i < S::NBARS; ++i) {
      const bool by_warps = (i >= S::SPLIT && i < S::SPLIT + B_NST) || i == S::A || i >= S::DRAIN;
      tc::mbar_init(BAR(i), by_warps ? F_NEPI : 1);
    }
    *abort_flag = 0;
    tc::fence_barrier_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  bool ok = true;

  if (warp == F_NEPI) {
    if (lane == 0) {
      auto wait = [&](int i, uint32_t par) {
        ok = ok && tc::mbar_wait_or_abort(BAR(i), par, abort_flag);
        return ok;
      };
      const float* dw_tile = p.dout + (int64_t)blockIdx.x * nch * WT_CHUNK;
      auto copy_chunk = [&](int k) {
        const int s = k % B_NST;
        const uint32_t st = base + s * S::STAGE;
        tc::mbar_expect_tx(BAR(S::LD + s), (WT_CHUNK + BIMG) * 4);
        tc::bulk_g2s(st, dw_tile + (int64_t)k * WT_CHUNK, WT_CHUNK * 4, BAR(S::LD + s));
        tc::bulk_g2s(st + 16384, p.tc_img_bwd + (int64_t)k * BIMG, BIMG * 4, BAR(S::LD + s));
      };
      constexpr uint32_t IDESC = tc::idesc_tf32(TM, H);
      constexpr uint32_t IDESC2 = tc::idesc_tf32(TM, 2 * H);  // B = the stacked hi|lo weight rows
      for (int k = 0; k < B_NST && k < nch; ++k) copy_chunk(k);
      for (int kc = 0; kc < nch; ++kc) {
        const int s = kc % B_NST;
        const int grp = kc / B_GROUP;
        if (!wait(S::SPLIT + s, (kc / B_NST) & 1)) break;
        // the previous group's partial sum has been drained into registers
        if (kc % B_GROUP == 0 && grp >= 1 && !wait(S::DRAIN + ((grp - 1) & 1), ((grp - 1) >> 1) & 1)) break;
        tc::fence_after_sync();
        const uint32_t ah = base + s * S::STAGE, al = tmem + B_ALO + 32 * s;  // A hi in smem, lo in TMEM
        const uint32_t bh = base + s * S::STAGE + 16384;  // hi rows [0, 64), lo rows [64, 128)
        const bool fresh = kc % B_GROUP == 0;
#pragma unroll
        for (int kb = 0; kb < KC / 8; ++kb) {
          const uint32_t off = kb * 32;
          // [A_hi B_hi | A_hi B_lo] into [0, 128), then A_lo B_hi into the small half
          tc::mma_tf32(tmem, tc::sw128_desc(ah + off), tc::sw128_desc(bh + off), IDESC2, !(fresh && kb == 0));
          tc::mma_tf32_ta(tmem + B_SMALL, al + kb * 8, tc::sw128_desc(bh + off), IDESC, 1);
        }
        tc::mma_commit(BAR(S::MMA + s));
        // stage (kc - 1) % B_NST (smem and TMEM) is free once MMA(kc - 1) is done, which
        // MMA(kc) queued behind it does not wait for: chunk kc - 1 + B_NST goes there
        if (kc >= 1 && kc - 1 + B_NST < nch) {
          if (!wait(S::MMA + (kc - 1) % B_NST, ((kc - 1) / B_NST) & 1)) break;
          copy_chunk(kc - 1 + B_NST);
        }
      }
      // every K-chunk MMA done before the hidden layers reuse stage memory and TMEM
      wait(S::MMA + (last % B_NST), (last / B_NST) & 1);
      uint32_t pa = 0, pacc = 0, ptl = 0;
      for (int j = nh - 1; j >= 1 && ok; --j) {
        tc::mbar_expect_tx(BAR(S::TL), IMG * 4);
        tc::bulk_g2s(base, p.tc_trunk_bwd + (int64_t)(j - 1) * IMG, IMG * 4, BAR(S::TL));
        if (!wait(S::A, pa) || !wait(S::TL, ptl)) break;
        pa ^= 1;
        ptl ^= 1;
        tc::fence_after_sync();
        mma_k64_split<H>(tmem, tmem + B_SMALL, tmem + B_TAHI, tmem + B_TALO, base, base + IMG * 2);
        tc::mma_commit(BAR(S::ACC));
        if (!wait(S::ACC, pacc)) break;  // the weight image is free again
        pacc ^= 1;
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3, g = warp >> 2;
    const int row = q * 32 + lane;
    const int64_t e = (int64_t)blockIdx.x * TM + row;
    const bool valid = e < p.E;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    auto wwait = [&](int i, uint32_t par) {
      const bool r = ok && tc::mbar_wait_or_abort(BAR(i), par, abort_flag);
      ok = __all_sync(0xffffffffu, r);
      return ok;
    };
    float* sW0 = reinterpret_cast<float*>(sm + S::W0);
    for (int i = t; i < NB * H / 4; i += 32 * F_NEPI)
      reinterpret_cast<float4*>(sW0)[i] = __ldg(reinterpret_cast<const float4*>(p.w[0]) + i);
    tc::named_sync(1, 32 * F_NEPI);
    // split each dW chunk into tf32 hi / lo, into TMEM; after the last chunk of
    // every group of B_GROUP chunks add the group's dH partial sum (this warp
    // group's 32 columns) into fp32 registers, so that no tensor-core
    // accumulator sums more than B_GROUP chunks
    float dh[32];
#pragma unroll
    for (int o = 0; o < 32; ++o) dh[o] = 0.f;
    // drain the group that ended at chunk kc_end (its MMAs have to be complete)
    auto drain = [&](int kc_end) {
      const int grp = kc_end / B_GROUP;
      if (!wwait(S::MMA + kc_end % B_NST, (kc_end / B_NST) & 1)) return false;
      tc::fence_after_sync();
      const uint32_t part_col = tmem + lane_base + 32 * g;
      tc::tmem_ld16_add(part_col + B_SMALL, dh);
      tc::tmem_ld16_add(part_col + B_SMALL + 16, dh + 16);
      tc::tmem_ld16_add(part_col, dh);
      tc::tmem_ld16_add(part_col + 16, dh + 16);
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(BAR(S::DRAIN + (grp & 1)));
      return true;
    };
    for (int kc = 0; kc < nch; ++kc) {
      const int s = kc % B_NST;
      if (!wwait(S::LD + s, (kc / B_NST) & 1)) break;
      unsigned char* src = sm + s * S::STAGE + row * 128;
      float v[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float4 x = *reinterpret_cast<const float4*>(src + (((4 * g + u) ^ (row & 7)) << 4));
        v[4 * u] = x.x;
        v[4 * u + 1] = x.y;
        v[4 * u + 2] = x.z;
        v[4 * u + 3] = x.w;
      }
      // hi part in place (the MMA's shared-memory A operand), lo part into TMEM
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<float4*>(src + (((4 * g + u) ^ (row & 7)) << 4)) =
            make_float4(tc::tf32_hi(v[4 * u]), tc::tf32_hi(v[4 * u + 1]), tc::tf32_hi(v[4 * u + 2]),
                        tc::tf32_hi(v[4 * u + 3]));
      float part[16];
#pragma unroll
      for (int o = 0; o < 16; ++o) part[o] = v[o] - tc::tf32_hi(v[o]);
      tc::tmem_st16(tmem + lane_base + B_ALO + 32 * s + 16 * g, part);
      tc::fence_proxy_async();  // the in-place hi values are read by the tensor core (async proxy)
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(BAR(S::SPLIT + s));
      // the previous group's partial sum, once this chunk is staged (overlaps its MMAs)
      if (kc >= 1 && (kc - 1) % B_GROUP == B_GROUP - 1 && !drain(kc - 1)) break;
    }
    if (ok) drain(last);
    // hidden layers nh-1 .. 1 on the tensor cores, this group's 32 columns
    uint32_t pacc = 0;
    for (int j = nh - 1; j >= 1 && ok; --j) {
      const float4* a4 = reinterpret_cast<const float4*>(p.act + e * (int64_t)(nh * H) + j * H + 32 * g);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) a = a4[k];
        dh[4 * k + 0] = valid ? dh[4 * k + 0] * silu_grad_f(a.x) : 0.f;
        dh[4 * k + 1] = valid ? dh[4 * k + 1] * silu_grad_f(a.y) : 0.f;
        dh[4 * k + 2] = valid ? dh[4 * k + 2] * silu_grad_f(a.z) : 0.f;
        dh[4 * k + 3] = valid ? dh[4 * k + 3] * silu_grad_f(a.w) : 0.f;
      }
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        float part[16];
#pragma unroll
        for (int o = 0; o < 16; ++o) part[o] = tc::tf32_hi(dh[16 * hf + o]);
        tc::tmem_st16(tmem + lane_base + B_TAHI + 32 * g + 16 * hf, part);
#pragma unroll
        for (int o = 0; o < 16; ++o) part[o] = dh[16 * hf + o] - tc::tf32_hi(dh[16 * hf + o]);
        tc::tmem_st16(tmem + lane_base + B_TALO + 32 * g + 16 * hf, part);
      }
      tc::tmem_wait_st();
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(BAR(S::A));
      if (!wwait(S::ACC, pacc)) break;
      pacc ^= 1;
      tc::fence_after_sync();
      tc::tmem_ld32(tmem + lane_base + 32 * g, dh);
      tc::tmem_wait_ld();
      tc::tmem_ld16_add(tmem + lane_base + B_SMALL + 32 * g, dh);
      tc::tmem_ld16_add(tmem + lane_base + B_SMALL + 32 * g + 16, dh + 16);
    }
    // layer 0 on the CUDA cores: dL/db[i] = sum_o dh[o] SiLU'(a0[o]) W0[i][o], the
    // two column halves added through shared memory
    float* sDb = reinterpret_cast<float*>(sm + S::DB);
    if (ok) {
      float da[32];
      const float4* a4 = reinterpret_cast<const float4*>(p.act + e * (int64_t)(nh * H) + 32 * g);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
        if (valid) a = a4[k];
        da[4 * k + 0] = dh[4 * k + 0] * silu_grad_f(a.x);
        da[4 * k + 1] = dh[4 * k + 1] * silu_grad_f(a.y);
        da[4 * k + 2] = dh[4 * k + 2] * silu_grad_f(a.z);
        da[4 * k + 3] = dh[4 * k + 3] * silu_grad_f(a.w);
      }
#pragma unroll
      for (int i = 0; i < NB; ++i) {
        const float4* w4 = reinterpret_cast<const float4*>(sW0 + i * H + 32 * g);
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float4 w = w4[k];
          acc = fmaf(da[4 * k + 0], w.x, acc);
          acc = fmaf(da[4 * k + 1], w.y, acc);
          acc = fmaf(da[4 * k + 2], w.z, acc);
          acc = fmaf(da[4 * k + 3], w.w, acc);
        }
        sDb[(row * 2 + g) * 16 + i] = acc;
      }
    }
    tc::named_sync(1, 32 * F_NEPI);
    if (ok && g == 0 && valid) {
#pragma unroll
      for (int i = 0; i < NB; ++i) p.db[e * NB + i] += sDb[(row * 2) * 16 + i] + sDb[(row * 2 + 1) * 16 + i];
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (!ok) atomicExch(p.err_flag, MLP_TC_TIMEOUT);
  if (warp == F_NEPI) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, F_TMEM);
  }
}

template <int NB>
int launch_fwd_nb(const MlpParams& p, cudaStream_t s) {
  const size_t smem = FwdSmem::REQUEST;
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_mlp_fwd_tc<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  // all of the SM's unified memory as shared memory: two CTAs per SM
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_mlp_fwd_tc<NB>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
  k_mlp_fwd_tc<NB><<<(unsigned)((p.E + TM - 1) / TM), F_NTHR, smem, s>>>(p);
  MACE_LAUNCH_CHECK("mlp_fwd_tc");
  return MACE_OK;
}

template <int NB>
int launch_bwd_nb(const MlpParams& p, cudaStream_t s) {
  const size_t smem = BwdSmem::REQUEST;
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_mlp_bwd_tc<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_mlp_bwd_tc<NB>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                     (int)cudaSharedmemCarveoutMaxShared));
  k_mlp_bwd_tc<NB><<<(unsigned)((p.E + TM - 1) / TM), F_NTHR, smem, s>>>(p);
  MACE_LAUNCH_CHECK("mlp_bwd_tc");
  return MACE_OK;
}

}  // namespace

bool mlp_tc_supported(const MlpParams& p) {
  if (!p.tc_img || !p.tc_img_bwd || !p.tc_trunk || !p.tc_trunk_bwd) return false;
  if (p.n_layers < 2) return false;
  const int nb = p.widths[0];
  if (nb != 4 && nb != 6 && nb != 8 && nb != 10 && nb != 12 && nb != 16) return false;
  for (int j = 1; j < p.n_layers; ++j)
    if (p.widths[j] != H) return false;
  return p.widths[p.n_layers] % 4 == 0;
}

int launch_mlp_fwd_tc(const MlpParams& p, cudaStream_t s) {
  switch (p.widths[0]) {
    case 4: return launch_fwd_nb<4>(p, s);
    case 6: return launch_fwd_nb<6>(p, s);
    case 8: return launch_fwd_nb<8>(p, s);
    case 10: return launch_fwd_nb<10>(p, s);
    case 12: return launch_fwd_nb<12>(p, s);
    default: return launch_fwd_nb<16>(p, s);
  }
}

int launch_mlp_bwd_tc(const MlpParams& p, cudaStream_t s) {
  switch (p.widths[0]) {
    case 4: return launch_bwd_nb<4>(p, s);
    case 6: return launch_bwd_nb<6>(p, s);
    case 8: return launch_bwd_nb<8>(p, s);
    case 10: return launch_bwd_nb<10>(p, s);
    case 12: return launch_bwd_nb<12>(p, s);
    default: return launch_bwd_nb<16>(p, s);
  }
}

}  // namespace mace
