// Radial MLP on the 5th-generation tensor cores (sm_100a tcgen05, kind::tf32
// with a 3-term hi/lo split for fp32-level accuracy; see tc.cuh).
//
// One CTA of 128 threads owns a tile of 128 edges; thread t owns edge t, which
// is also TMEM lane t of every 128-row accumulator.  About 100 KB of shared
// memory, so two CTAs share an SM and overlap each other's phases.
//
// Forward:
//   layer 0 (radial features -> 64) on the CUDA cores; every 64 x 64 hidden
//   layer and every 64-column chunk of the last layer as 8 K-blocks x 3
//   tcgen05.mma (M = 128, N = 64, K = 8) from the swizzled hi/lo activation
//   tile (A) and a pre-split, pre-swizzled weight image (B) brought in by a
//   1-D bulk copy; epilogues read TMEM per edge (pre-activations stored for
//   the backward, SiLU, split, back to A).  Two TMEM buffers alternate
//   between chunks; the next image is fetched while an epilogue runs.
// Backward:
//   dH = dW (128 x W) . W_last^T with a 2-stage pipeline (the next dW chunk
//   is prefetched into registers while the current one is split into A and
//   its MMAs run), then for every hidden layer dH <- (dH * SiLU'(a)) . W_j^T
//   on the tensor cores, and the last step to dL/db on the CUDA cores.
//
// Every mbarrier wait is bounded (tc::mbar_wait gives up after ~2 s); on a
// timeout the kernel records MLP_TC_TIMEOUT in the error flag, frees its TMEM
// and returns.
#include "common.cuh"
#include "tc.cuh"

namespace mace {

namespace {

constexpr int TM = 128;   // edges per tile (MMA M)
constexpr int H = 64;     // hidden width
constexpr int TN = 64;    // output columns per forward chunk (MMA N)
constexpr int KC = 32;    // backward K chunk (one 128-byte panel)
constexpr int MLP_TC_TIMEOUT = 2;
constexpr int IMG = 2 * 64 * 64;  // floats of one 64 x 64 hi/lo image

__device__ __forceinline__ void put_hilo(unsigned char* a_hi, unsigned char* a_lo, int row, int k0, float4 v) {
  float4 hi, lo;
  hi.x = tc::tf32_hi(v.x);
  hi.y = tc::tf32_hi(v.y);
  hi.z = tc::tf32_hi(v.z);
  hi.w = tc::tf32_hi(v.w);
  lo.x = v.x - hi.x;
  lo.y = v.y - hi.y;
  lo.z = v.z - hi.z;
  lo.w = v.w - hi.w;
  const uint32_t off = tc::sw128_offset(row, k0, TM);
  *reinterpret_cast<float4*>(a_hi + off) = hi;
  *reinterpret_cast<float4*>(a_lo + off) = lo;
}

// D (128 x N) = A (128 x 64, hi/lo) . B (N x 64, hi/lo)^T, issued by one thread
template <int N>
__device__ __forceinline__ void mma_k64(uint32_t tmem, uint32_t a_hi, uint32_t a_lo, uint32_t b_hi, uint32_t b_lo) {
  constexpr uint32_t IDESC = tc::idesc_tf32(TM, N);
#pragma unroll
  for (int kb = 0; kb < H / 8; ++kb) {
    const uint32_t oa = (kb >> 2) * (TM * 128) + (kb & 3) * 32;
    const uint32_t ob = (kb >> 2) * (N * 128) + (kb & 3) * 32;
    tc::mma_tf32(tmem, tc::sw128_desc(a_hi + oa), tc::sw128_desc(b_hi + ob), IDESC, kb > 0);
    tc::mma_tf32(tmem, tc::sw128_desc(a_hi + oa), tc::sw128_desc(b_lo + ob), IDESC, 1);
    tc::mma_tf32(tmem, tc::sw128_desc(a_lo + oa), tc::sw128_desc(b_hi + ob), IDESC, 1);
  }
}

__device__ __forceinline__ void tmem_row64(uint32_t tmem, int warp, int col0, float* v) {
  tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + col0, v);
  tc::tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + col0 + 32, v + 32);
  tc::tmem_wait_ld();
}

struct FwdSmem {
  static constexpr int A_HI = 0;                   // 128 x 64 fp32 = 32 KB
  static constexpr int A_LO = A_HI + TM * H * 4;   // 32 KB
  static constexpr int B = A_LO + TM * H * 4;      // hi/lo image, 32 KB
  static constexpr int W0 = B + IMG * 4;           // layer 0 weights, <= 16 x 64
  static constexpr int BARS = W0 + 16 * H * 4;
  static constexpr int TOTAL = BARS + 64;
};

template <int NB>
__global__ void __launch_bounds__(128, 2) k_mlp_fwd_tc(MlpParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + FwdSmem::BARS);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + FwdSmem::BARS + 32);
  float* sW0 = reinterpret_cast<float*>(sm + FwdSmem::W0);
  unsigned char* a_hi_p = sm + FwdSmem::A_HI;
  unsigned char* a_lo_p = sm + FwdSmem::A_LO;
  const uint32_t bar_b = tc::smem_u32(&bars[0]);
  const uint32_t bar_m = tc::smem_u32(&bars[1]);
  const uint32_t a_hi = tc::smem_u32(a_hi_p), a_lo = tc::smem_u32(a_lo_p);
  const uint32_t b_hi = tc::smem_u32(sm + FwdSmem::B), b_lo = b_hi + IMG * 2;
  const int t = threadIdx.x, warp = t >> 5;
  const int64_t e = (int64_t)blockIdx.x * TM + t;
  const bool valid = e < p.E;
  const int nh = p.n_layers - 1;
  const int wout = p.widths[p.n_layers];
  const int nchunk = (wout + TN - 1) / TN;
  const int n_img = (nh - 1) + nchunk;  // images in order: hidden 1.., then last-layer chunks
  auto image = [&](int i) -> const float* {
    return i < nh - 1 ? p.tc_trunk + (int64_t)i * IMG : p.tc_img + (int64_t)(i - (nh - 1)) * IMG;
  };

  if (warp == 0) {
    tc::tmem_alloc(tc::smem_u32(tslot), 2 * TN);
    tc::tmem_relinquish();
  }
  if (t == 0) {
    tc::mbar_init(bar_b, 1);
    tc::mbar_init(bar_m, 1);
    tc::fence_barrier_init();
  }
  for (int q = t; q < NB * H; q += TM) sW0[q] = __ldg(p.w[0] + q);
  __syncthreads();
  if (t == 0) {  // first image in flight during layer 0
    tc::mbar_expect_tx(bar_b, IMG * 4);
    tc::bulk_g2s(b_hi, image(0), IMG * 4, bar_b);
  }
  // ---- layer 0 on the CUDA cores ----
  float y[H];
  {
    float x[NB];
#pragma unroll
    for (int i = 0; i < NB; ++i) x[i] = valid ? p.b[e * NB + i] : 0.f;
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
  const uint32_t tmem = *tslot;
  uint32_t pb = 0, pm = 0;
  bool ok = true;
  for (int j = 0; j < nh && ok; ++j) {
    // epilogue of hidden layer j: store pre-activation, SiLU, split into A
    if (valid) {
      float4* act = reinterpret_cast<float4*>(p.act + e * (int64_t)(nh * H) + j * H);
#pragma unroll
      for (int q = 0; q < H / 4; ++q) act[q] = make_float4(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]);
    }
#pragma unroll
    for (int q = 0; q < H / 4; ++q) {
      float4 h = valid ? make_float4(silu_f(y[4 * q]), silu_f(y[4 * q + 1]), silu_f(y[4 * q + 2]), silu_f(y[4 * q + 3]))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
      put_hilo(a_hi_p, a_lo_p, t, 4 * q, h);
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    if (j == nh - 1) break;  // the last hidden activation feeds the output chunks
    // hidden layer j+1 on the tensor cores (TMEM buffer 0)
    if (t == 0) {
      ok = tc::mbar_wait(bar_b, pb);
      if (ok) {
        tc::fence_after_sync();
        mma_k64<TN>(tmem, a_hi, a_lo, b_hi, b_lo);
        tc::mma_commit(bar_m);
      }
    }
    pb ^= 1;
    ok = tc::mbar_wait(bar_m, pm) && ok;
    pm ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc::fence_after_sync();
    if (t == 0) {  // B is free again: fetch the next image
      tc::mbar_expect_tx(bar_b, IMG * 4);
      tc::bulk_g2s(b_hi, image(j + 1), IMG * 4, bar_b);
    }
    tmem_row64(tmem, warp, 0, y);
  }
  // ---- last layer: 64-column chunks, TMEM buffers alternate ----
  for (int c = 0; c < nchunk && ok; ++c) {
    const uint32_t buf = tmem + (c & 1) * TN;
    if (t == 0) {
      ok = tc::mbar_wait(bar_b, pb);
      if (ok) {
        tc::fence_after_sync();
        mma_k64<TN>(buf, a_hi, a_lo, b_hi, b_lo);
        tc::mma_commit(bar_m);
      }
    }
    pb ^= 1;
    ok = tc::mbar_wait(bar_m, pm) && ok;
    pm ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc::fence_after_sync();
    const int next = (nh - 1) + c + 1;
    if (t == 0 && next < n_img) {
      tc::mbar_expect_tx(bar_b, IMG * 4);
      tc::bulk_g2s(b_hi, image(next), IMG * 4, bar_b);
    }
    float v[TN];
    tmem_row64(buf, warp, 0, v);
    if (valid) {
      float* dst = p.out + e * (int64_t)wout + c * TN;
#pragma unroll
      for (int q = 0; q < TN / 4; ++q)
        if (c * TN + 4 * q < wout)
          *reinterpret_cast<float4*>(dst + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    tc::fence_before_sync();
  }
  if (!ok && t == 0) atomicExch(p.err_flag, MLP_TC_TIMEOUT);
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, 2 * TN);
}

struct BwdSmem {
  static constexpr int A = 0;                         // [2 stages][hi, lo] 128 x 32 = 16 KB each (64 KB)
  static constexpr int B = A + 2 * 2 * TM * KC * 4;   // [2 stages][hi, lo] 64 x 32 = 8 KB each (32 KB)
  static constexpr int W0 = B + 2 * 2 * H * KC * 4;   // layer 0 weights (in, out) <= 16 x 64
  static constexpr int BARS = W0 + 16 * H * 4;
  static constexpr int TOTAL = BARS + 128;
};

template <int NB>
__global__ void __launch_bounds__(128, 2) k_mlp_bwd_tc(MlpParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + BwdSmem::BARS);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + BwdSmem::BARS + 64);
  float* sW0 = reinterpret_cast<float*>(sm + BwdSmem::W0);
  const int t = threadIdx.x, warp = t >> 5;
  const int64_t e = (int64_t)blockIdx.x * TM + t;
  const bool valid = e < p.E;
  const int nh = p.n_layers - 1;
  const int wout = p.widths[p.n_layers];
  const uint32_t bar_b[2] = {tc::smem_u32(&bars[0]), tc::smem_u32(&bars[1])};
  const uint32_t bar_m[2] = {tc::smem_u32(&bars[2]), tc::smem_u32(&bars[3])};
  const uint32_t bar_tb = tc::smem_u32(&bars[4]), bar_tm = tc::smem_u32(&bars[5]);
  if (warp == 0) {
    tc::tmem_alloc(tc::smem_u32(tslot), H);
    tc::tmem_relinquish();
  }
  if (t == 0) {
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(bar_b[i], 1);
      tc::mbar_init(bar_m[i], 1);
    }
    tc::mbar_init(bar_tb, 1);
    tc::mbar_init(bar_tm, 1);
    tc::fence_barrier_init();
  }
  for (int q = t; q < NB * H; q += TM) sW0[q] = __ldg(p.w[0] + q);  // (in = NB, out = 64)
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tslot;
  constexpr uint32_t IDESC = tc::idesc_tf32(TM, H);
  const int nchunk = (wout + KC - 1) / KC;
  const float* row = p.dout + e * (int64_t)wout;
  auto load_chunk = [&](int kc, float4* r) {
#pragma unroll
    for (int q = 0; q < KC / 4; ++q) {
      const int c = kc * KC + 4 * q;
      r[q] = (valid && c < wout) ? __ldg(reinterpret_cast<const float4*>(row + c)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float4 cur[KC / 4], nxt[KC / 4];
  load_chunk(0, cur);
  bool ok = true;
  for (int kc = 0; kc < nchunk; ++kc) {
    const int s = kc & 1;
    unsigned char* a_hi_p = sm + BwdSmem::A + (s * 2 + 0) * TM * KC * 4;
    unsigned char* a_lo_p = sm + BwdSmem::A + (s * 2 + 1) * TM * KC * 4;
    const uint32_t b_hi = tc::smem_u32(sm + BwdSmem::B + (s * 2 + 0) * H * KC * 4);
    const uint32_t b_lo = b_hi + H * KC * 4;
    if (kc >= 2) ok = tc::mbar_wait(bar_m[s], ((kc - 2) >> 1) & 1) && ok;  // stage s free again
    if (t == 0 && ok) {
      tc::mbar_expect_tx(bar_b[s], 2 * H * KC * 4);
      tc::bulk_g2s(b_hi, p.tc_img_bwd + (int64_t)kc * 2 * H * KC, 2 * H * KC * 4, bar_b[s]);
    }
#pragma unroll
    for (int q = 0; q < KC / 4; ++q) {
      const float4 v = cur[q];
      float4 hi, lo;
      hi.x = tc::tf32_hi(v.x);
      hi.y = tc::tf32_hi(v.y);
      hi.z = tc::tf32_hi(v.z);
      hi.w = tc::tf32_hi(v.w);
      lo.x = v.x - hi.x;
      lo.y = v.y - hi.y;
      lo.z = v.z - hi.z;
      lo.w = v.w - hi.w;
      const uint32_t off = tc::sw128_offset(t, 4 * q, TM);
      *reinterpret_cast<float4*>(a_hi_p + off) = hi;
      *reinterpret_cast<float4*>(a_lo_p + off) = lo;
    }
    if (kc + 1 < nchunk) load_chunk(kc + 1, nxt);
    tc::fence_proxy_async();
    ok = __syncthreads_and(ok);
    if (!ok) break;
    if (t == 0) {
      ok = tc::mbar_wait(bar_b[s], (kc >> 1) & 1);
      if (ok) {
        tc::fence_after_sync();
        const uint32_t a_hi = tc::smem_u32(a_hi_p), a_lo = tc::smem_u32(a_lo_p);
#pragma unroll
        for (int kb = 0; kb < KC / 8; ++kb) {
          const uint32_t off = kb * 32;
          tc::mma_tf32(tmem, tc::sw128_desc(a_hi + off), tc::sw128_desc(b_hi + off), IDESC, (kc > 0 || kb > 0));
          tc::mma_tf32(tmem, tc::sw128_desc(a_hi + off), tc::sw128_desc(b_lo + off), IDESC, 1);
          tc::mma_tf32(tmem, tc::sw128_desc(a_lo + off), tc::sw128_desc(b_hi + off), IDESC, 1);
        }
        tc::mma_commit(bar_m[s]);
      }
    }
#pragma unroll
    for (int q = 0; q < KC / 4; ++q) cur[q] = nxt[q];
  }
  float dh[H];
  if (ok) {
    const int last = nchunk - 1;
    ok = tc::mbar_wait(bar_m[last & 1], (last >> 1) & 1);
    ok = __syncthreads_and(ok);
  }
  if (ok) {
    tc::fence_after_sync();
    tmem_row64(tmem, warp, 0, dh);
  }
  // ---- hidden layers nh-1 .. 1 on the tensor cores ----
  unsigned char* a_hi_p = sm + BwdSmem::A;               // 128 x 64 hi (32 KB)
  unsigned char* a_lo_p = sm + BwdSmem::A + TM * H * 4;  // 128 x 64 lo (32 KB)
  const uint32_t b_hi = tc::smem_u32(sm + BwdSmem::B), b_lo = b_hi + IMG * 2;
  uint32_t ptb = 0, ptm = 0;
  for (int j = nh - 1; j >= 1 && ok; --j) {
    if (t == 0) {
      tc::mbar_expect_tx(bar_tb, IMG * 4);
      tc::bulk_g2s(b_hi, p.tc_trunk_bwd + (int64_t)(j - 1) * IMG, IMG * 4, bar_tb);
    }
    const float4* a4 = reinterpret_cast<const float4*>(p.act + e * (int64_t)(nh * H) + j * H);
#pragma unroll
    for (int q = 0; q < H / 4; ++q) {
      float4 a = valid ? a4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 d = make_float4(dh[4 * q] * silu_grad_f(a.x), dh[4 * q + 1] * silu_grad_f(a.y),
                             dh[4 * q + 2] * silu_grad_f(a.z), dh[4 * q + 3] * silu_grad_f(a.w));
      if (!valid) d = make_float4(0.f, 0.f, 0.f, 0.f);
      put_hilo(a_hi_p, a_lo_p, t, 4 * q, d);
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    if (t == 0) {
      ok = tc::mbar_wait(bar_tb, ptb);
      if (ok) {
        tc::fence_after_sync();
        mma_k64<H>(tmem, tc::smem_u32(a_hi_p), tc::smem_u32(a_lo_p), b_hi, b_lo);
        tc::mma_commit(bar_tm);
      }
    }
    ptb ^= 1;
    ok = tc::mbar_wait(bar_tm, ptm) && ok;
    ptm ^= 1;
    ok = __syncthreads_and(ok);
    if (!ok) break;
    tc::fence_after_sync();
    tmem_row64(tmem, warp, 0, dh);
    tc::fence_before_sync();
    __syncthreads();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, H);
  if (!ok) {
    if (t == 0) atomicExch(p.err_flag, MLP_TC_TIMEOUT);
    return;
  }
  // ---- layer 0 on the CUDA cores: dL/db[i] = sum_o dh[o] SiLU'(a0[o]) W0[i][o] ----
  if (!valid) return;
  float da[H];
  const float4* a4 = reinterpret_cast<const float4*>(p.act + e * (int64_t)(nh * H));
#pragma unroll
  for (int q = 0; q < H / 4; ++q) {
    const float4 a = a4[q];
    da[4 * q + 0] = dh[4 * q + 0] * silu_grad_f(a.x);
    da[4 * q + 1] = dh[4 * q + 1] * silu_grad_f(a.y);
    da[4 * q + 2] = dh[4 * q + 2] * silu_grad_f(a.z);
    da[4 * q + 3] = dh[4 * q + 3] * silu_grad_f(a.w);
  }
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    const float4* w4 = reinterpret_cast<const float4*>(sW0 + i * H);
    float acc = 0.f;
#pragma unroll
    for (int q = 0; q < H / 4; ++q) {
      const float4 w = w4[q];
      acc = fmaf(da[4 * q + 0], w.x, acc);
      acc = fmaf(da[4 * q + 1], w.y, acc);
      acc = fmaf(da[4 * q + 2], w.z, acc);
      acc = fmaf(da[4 * q + 3], w.w, acc);
    }
    p.db[e * NB + i] += acc;
  }
}

template <int NB>
int launch_fwd_nb(const MlpParams& p, cudaStream_t s) {
  const size_t smem = FwdSmem::TOTAL + 1024;
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_mlp_fwd_tc<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_mlp_fwd_tc<NB><<<(unsigned)((p.E + TM - 1) / TM), TM, smem, s>>>(p);
  MACE_LAUNCH_CHECK("mlp_fwd_tc");
  return MACE_OK;
}

template <int NB>
int launch_bwd_nb(const MlpParams& p, cudaStream_t s) {
  const size_t smem = BwdSmem::TOTAL + 1024;
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_mlp_bwd_tc<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_mlp_bwd_tc<NB><<<(unsigned)((p.E + TM - 1) / TM), TM, smem, s>>>(p);
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
