// Interaction message passing: channelwise (uvu) tensor product of the sender's
// up-projected features with the edge spherical harmonics, weighted by the
// per-edge radial-MLP output, summed over the receiver's incoming edges.
//
// Reference: conv_tp + scatter_sum in blocks.py:242-279 with the uvu
// semantics of tensor_product.py:833-1043 (instructions from utils.py:87-156):
//   A[n][k][u, m] = sum_{e -> n} w_e[k, u] * sum_{i, j} pw_k CG_k[i, j, m] x1[s_e][u, i] Y_e[j]
//
// Design: one CTA per receiver node, one thread per channel u.  Edges are
// receiver-sorted (CSR), so the scatter is a segmented sum done in registers
// and written once: the per-edge message (E x 5120 floats for the medium
// model) never exists in memory.  The CG contraction is re-associated per
// edge as M_k[i][m] = sum_j pw_k CG_k[i, j, m] Y_e[j] (shared by all channels,
// staged in shared memory), leaving (2l1+1)(2l3+1) FMAs per channel.
//
// Backward (same CTA layout) produces, deterministically and without atomics:
//   dw_e[k, u]         (input of the radial-MLP backward)
//   dY_e[j]            (block reduction over channels)
//   d up[n]            through the reverse edge rev(e) = (n -> s_e, -S), whose
//                      weights equal w_e and whose SH equal (-1)^l2 Y_e bitwise,
//                      so the sender-side sum of node n is a sum over n's own
//                      incoming edges reading dA of the neighbour.
#include "common.cuh"

namespace mace {

namespace {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ int cdim(int l) { return 2 * l + 1; }

// ---------------------------------------------------------------------------
// per-chunk staging: senders, SH rows, and M rows for all slots
// ---------------------------------------------------------------------------
__device__ void stage_chunk(const ConvParams& p, int64_t cb, int ne, int* sSnd, float* sY,
                            float* sM) {
  const int tid = threadIdx.x, nt = blockDim.x;
  for (int j = tid; j < ne; j += nt) sSnd[j] = p.snd[cb + j];
  for (int q = tid; q < ne * 16; q += nt) sY[q] = p.Y[cb * 16 + q];
  __syncthreads();
  for (int k = 0; k < p.n_mid; ++k) {
    const ConvSlotDev& sl = p.slot[k];
    const int D1 = cdim(sl.l1), D2 = cdim(sl.l2), D3 = cdim(sl.l3);
    const int sz = D1 * D3, yo = sl.l2 * sl.l2;
    for (int idx = tid; idx < ne * sz; idx += nt) {
      int j = idx / sz, q = idx % sz;
      int i = q / D3, m = q % D3;
      const float* y = sY + j * 16 + yo;
      float acc = 0.f;
      for (int jj = 0; jj < D2; ++jj) acc = fmaf(__ldg(sl.cg + (i * D2 + jj) * D3 + m), y[jj], acc);
      sM[j * p.m_tot + sl.m_off + q] = acc;
    }
  }
  __syncthreads();
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------
template <int D1, int D3>
__device__ __forceinline__ void fwd_slot(const ConvParams& p, const ConvSlotDev& sl, int k,
                                         int64_t n, int64_t cb, int ne, bool first,
                                         const int* sSnd, const float* sM) {
  const int u = threadIdx.x;
  const int C = p.C;
  float acc[D3];
  float* out = p.A + n * p.mid_dim + sl.off + u;
#pragma unroll
  for (int m = 0; m < D3; ++m) acc[m] = first ? 0.f : out[m * C];
  for (int j = 0; j < ne; ++j) {
    const int64_t s = sSnd[j];
    const float* x = p.up + s * p.in_dim + sl.src_off + u;
    float x1[D1];
#pragma unroll
    for (int i = 0; i < D1; ++i) x1[i] = __ldg(x + i * C);
    const float w = __ldg(p.w + wt_index(cb + j - p.e0, k * C + u, p.wnch));
    const float* Mk = sM + j * p.m_tot + sl.m_off;
#pragma unroll
    for (int m = 0; m < D3; ++m) {
      float t = 0.f;
#pragma unroll
      for (int i = 0; i < D1; ++i) t = fmaf(x1[i], Mk[i * D3 + m], t);
      acc[m] = fmaf(w, t, acc[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < D3; ++m) out[m * C] = acc[m];
}

__global__ void k_conv_fwd(ConvParams p, int EC) {
  extern __shared__ float sm[];
  int* sSnd = reinterpret_cast<int*>(sm);
  float* sY = sm + EC;
  float* sM = sY + EC * 16;
  const int64_t n = p.n0 + blockIdx.x;
  if (conv_receiver_skipped(p, n)) return;  // the other part of a split launch
  const int64_t e_beg = p.row_ptr[n], e_end = p.row_ptr[n + 1];
  if (e_beg == e_end) {
    for (int q = threadIdx.x; q < p.mid_dim; q += blockDim.x) p.A[n * p.mid_dim + q] = 0.f;
    return;
  }
  for (int64_t cb = e_beg; cb < e_end; cb += EC) {
    const int ne = (int)imin64(EC, e_end - cb);
    stage_chunk(p, cb, ne, sSnd, sY, sM);
    const bool first = (cb == e_beg);
    for (int k = 0; k < p.n_mid; ++k) {
      const ConvSlotDev& sl = p.slot[k];
      switch (sl.l1 * 4 + sl.l3) {
#define FWD_CASE(a, b) \
  case a * 4 + b: fwd_slot<2 * a + 1, 2 * b + 1>(p, sl, k, n, cb, ne, first, sSnd, sM); break;
        FWD_CASE(0, 0) FWD_CASE(0, 1) FWD_CASE(0, 2) FWD_CASE(0, 3)
        FWD_CASE(1, 0) FWD_CASE(1, 1) FWD_CASE(1, 2) FWD_CASE(1, 3)
        FWD_CASE(2, 0) FWD_CASE(2, 1) FWD_CASE(2, 2) FWD_CASE(2, 3)
#undef FWD_CASE
        default: break;
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------

// Sum 16 per-lane values over the warp; lane L ends with the total of index L>>1.
__device__ __forceinline__ float warp_reduce16(float s[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool hi = lane & 16;
    float keep = hi ? s[8 + i] : s[i];
    float send = hi ? s[i] : s[8 + i];
    s[i] = keep + __shfl_xor_sync(FULL, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 8;
    float keep = hi ? s[4 + i] : s[i];
    float send = hi ? s[i] : s[4 + i];
    s[i] = keep + __shfl_xor_sync(FULL, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 4;
    float keep = hi ? s[2 + i] : s[i];
    float send = hi ? s[i] : s[2 + i];
    s[i] = keep + __shfl_xor_sync(FULL, send, 4);
  }
  {
    const bool hi = lane & 2;
    float keep = hi ? s[1] : s[0];
    float send = hi ? s[0] : s[1];
    s[0] = keep + __shfl_xor_sync(FULL, send, 2);
  }
  return s[0] + __shfl_xor_sync(FULL, s[0], 1);
}

// Per receiver n, slot k and channel u the receiver's gradient enters every edge
// only through H[i][j] = sum_m pw CG[i, j, m] dA[n][k][m][u]; it is formed once
// per CTA, so each edge needs (2l1+1)(2l2+1) multiply-adds per channel for
//   dw_e[k, u] = sum_{i,j} x1[i] H[i][j] Y_e[j]     and     dY_e[j] += w sum_i x1[i] H[i][j].
template <int L1, int L2, int L3>
__device__ __forceinline__ void bwd_slot(const ConvParams& p, const ConvSlotDev& sl, int k,
                                         int64_t e, int s, const float* Mk, const float* Ye,
                                         const float* sH, float* sDup, float sdy[16], int u) {
  constexpr int D1 = 2 * L1 + 1, D2 = 2 * L2 + 1, D3 = 2 * L3 + 1, YO = L2 * L2;
  constexpr float PAR = (L2 & 1) ? -1.f : 1.f;
  const int C = p.C;
  const float* x = p.up + (int64_t)s * p.in_dim + sl.src_off + u;
  float x1[D1];
#pragma unroll
  for (int i = 0; i < D1; ++i) x1[i] = __ldg(x + i * C);
  const float w = __ldg(p.w + wt_index(e - p.e0, k * C + u, p.wnch));
  float gr[D3];
  const float* dAs = p.dA + (int64_t)s * p.mid_dim + sl.off + u;
#pragma unroll
  for (int m = 0; m < D3; ++m) gr[m] = __ldg(dAs + m * C);
  const float* H = sH + sl.h_off * C + u;
  float xh[D2];
#pragma unroll
  for (int jj = 0; jj < D2; ++jj) xh[jj] = 0.f;
#pragma unroll
  for (int i = 0; i < D1; ++i)
#pragma unroll
    for (int jj = 0; jj < D2; ++jj) xh[jj] = fmaf(x1[i], H[(i * D2 + jj) * C], xh[jj]);
  float dw = 0.f;
#pragma unroll
  for (int jj = 0; jj < D2; ++jj) {
    dw = fmaf(xh[jj], Ye[YO + jj], dw);
    sdy[YO + jj] = fmaf(w, xh[jj], sdy[YO + jj]);
  }
  p.dw[wt_index(e - p.e0, k * C + u, p.wnch)] = dw;
  // sender side of node n through the reverse edge
#pragma unroll
  for (int i = 0; i < D1; ++i) {
    float r = 0.f;
#pragma unroll
    for (int m = 0; m < D3; ++m) r = fmaf(Mk[i * D3 + m], gr[m], r);
    sDup[(sl.src_ch + i) * C + u] += PAR * w * r;
  }
}

// G groups of C threads share one receiver: group g takes edges j = g, g+G, ...
// of every chunk, so the per-receiver tables (H, M rows) are staged once for
// G times as many warps.
__global__ void __launch_bounds__(512, 2) k_conv_bwd(ConvParams p, int EC, int G) {
  extern __shared__ float sm[];
  const int C = p.C;
  const int nw = C / 32;                   // warps per group
  int* sSnd = reinterpret_cast<int*>(sm);
  float* sY = sm + EC;
  float* sM = sY + EC * 16;
  float* sRed = sM + EC * p.m_tot;        // nw x EC x 16
  float* sH = sRed + nw * EC * 16;         // h_tot x C
  float* sDupAll = sH + p.h_tot * C;       // G x in_dim
  const int64_t n = p.n0 + blockIdx.x;
  if (conv_receiver_skipped(p, n)) return;  // the other part of a split launch
  const int tid = threadIdx.x;
  const int u = tid % C, grp = tid / C;
  float* sDup = sDupAll + grp * p.in_dim;
  const int64_t e_beg = p.row_ptr[n], e_end = p.row_ptr[n + 1];
  for (int q = tid; q < G * p.in_dim; q += blockDim.x) sDupAll[q] = 0.f;
  // H_k[i][j] = sum_m pw CG_k[i, j, m] dA[n][k][m][u] (thread u's own column), slots split over groups
  {
    const float* g = p.dA + n * p.mid_dim + u;
    for (int k = grp; k < p.n_mid; k += G) {
      const ConvSlotDev& sl = p.slot[k];
      const int D1 = cdim(sl.l1), D2 = cdim(sl.l2), D3 = cdim(sl.l3);
      float gk[7];
#pragma unroll
      for (int m = 0; m < 7; ++m) gk[m] = (m < D3) ? g[sl.off + m * C] : 0.f;
      for (int i = 0; i < D1; ++i)
        for (int jj = 0; jj < D2; ++jj) {
          float a = 0.f;
#pragma unroll
          for (int m = 0; m < 7; ++m)
            if (m < D3) a = fmaf(__ldg(sl.cg + (i * D2 + jj) * D3 + m), gk[m], a);
          sH[(sl.h_off + i * D2 + jj) * C + u] = a;
        }
    }
  }
  __syncthreads();
  const int warp = u >> 5, lane = tid & 31;
  for (int64_t cb = e_beg; cb < e_end; cb += EC) {
    const int ne = (int)imin64(EC, e_end - cb);
    stage_chunk(p, cb, ne, sSnd, sY, sM);
    for (int j = grp; j < ne; j += G) {
      float sdy[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) sdy[q] = 0.f;
      const int s = sSnd[j];
      const int64_t e = cb + j;
      const float* Mrow = sM + j * p.m_tot;
      const float* Ye = sY + j * 16;
      for (int k = 0; k < p.n_mid; ++k) {
        const ConvSlotDev& sl = p.slot[k];
        const float* Mk = Mrow + sl.m_off;
        switch (sl.combo) {
#define BWD_CASE(a, b, c) \
  case a * 16 + b * 4 + c: bwd_slot<a, b, c>(p, sl, k, e, s, Mk, Ye, sH, sDup, sdy, u); break;
          BWD_CASE(0, 0, 0) BWD_CASE(0, 1, 1) BWD_CASE(0, 2, 2) BWD_CASE(0, 3, 3)
          BWD_CASE(1, 0, 1) BWD_CASE(1, 1, 0) BWD_CASE(1, 1, 1) BWD_CASE(1, 1, 2)
          BWD_CASE(1, 2, 1) BWD_CASE(1, 2, 2) BWD_CASE(1, 2, 3) BWD_CASE(1, 3, 2)
          BWD_CASE(1, 3, 3)
          BWD_CASE(2, 0, 2) BWD_CASE(2, 1, 1) BWD_CASE(2, 1, 2) BWD_CASE(2, 1, 3)
          BWD_CASE(2, 2, 0) BWD_CASE(2, 2, 1) BWD_CASE(2, 2, 2) BWD_CASE(2, 2, 3)
          BWD_CASE(2, 3, 1) BWD_CASE(2, 3, 2) BWD_CASE(2, 3, 3)
#undef BWD_CASE
          default: break;
        }
      }
      float tot = warp_reduce16(sdy);
      if ((lane & 1) == 0) sRed[(warp * EC + j) * 16 + (lane >> 1)] = tot;
    }
    __syncthreads();
    for (int idx = tid; idx < ne * 16; idx += blockDim.x) {
      const int j = idx >> 4, q = idx & 15;
      float v = 0.f;
      for (int w = 0; w < nw; ++w) v += sRed[(w * EC + j) * 16 + q];
      p.dY[(cb + j) * 16 + q] += v;
    }
    __syncthreads();
  }
  for (int q = tid; q < p.in_dim; q += blockDim.x) {
    float v = 0.f;
    for (int g = 0; g < G; ++g) v += sDupAll[g * p.in_dim + q];  // fixed order: deterministic
    p.dup[n * p.in_dim + q] = v;
  }
}

}  // namespace

static int conv_check(const ConvParams& p) {
  if (p.C % 32 != 0 || p.C > 1024) return fail(MACE_ERR_UNSUPPORTED, "channels must be a multiple of 32");
  for (int k = 0; k < p.n_mid; ++k) {
    const ConvSlotDev& s = p.slot[k];
    if (s.l1 > 2 || s.l2 > 3 || s.l3 > 3)
      return fail(MACE_ERR_UNSUPPORTED, "conv_tp supports l1 <= 2, l2 <= 3, l3 <= 3");
  }
  return MACE_OK;
}

// receivers n0 .. N-1 (p.N is the end of the range)
int launch_conv_fwd(const ConvParams& p, cudaStream_t s) {
  if (p.N <= p.n0) return MACE_OK;
  int rc = conv_check(p);
  if (rc) return rc;
  bool used = false;
  rc = launch_conv_fwd_sig(p, s, &used);
  if (rc || used) return rc;
  const int EC = 64;
  size_t smem = (size_t)(EC + EC * 16 + EC * p.m_tot) * sizeof(float);
  if (smem > 48 * 1024)
    MACE_CUDA_TRY(cudaFuncSetAttribute(k_conv_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_conv_fwd<<<(unsigned)(p.N - p.n0), p.C, smem, s>>>(p, EC);
  MACE_LAUNCH_CHECK("conv_fwd");
  return MACE_OK;
}

int launch_conv_bwd(const ConvParams& p, cudaStream_t s, bool* need_gather) {
  *need_gather = false;
  if (p.N <= p.n0) return MACE_OK;
  int rc = conv_check(p);
  if (rc) return rc;
  bool used = false;
  rc = launch_conv_bwd_sig(p, s, &used, need_gather);
  if (rc || used) return rc;
  const int EC = 32;
  const int nw = p.C / 32;
  int G = 1024 / p.C;
  if (G > 4) G = 4;
  size_t smem = (size_t)(EC + EC * 16 + EC * p.m_tot + nw * EC * 16 + p.h_tot * p.C + G * p.in_dim) * sizeof(float);
  if (smem > 227 * 1024) return fail(MACE_ERR_UNSUPPORTED, "conv backward tile exceeds shared memory");
  if (smem > 48 * 1024)
    MACE_CUDA_TRY(cudaFuncSetAttribute(k_conv_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_conv_bwd<<<(unsigned)(p.N - p.n0), p.C * G, smem, s>>>(p, EC, G);
  MACE_LAUNCH_CHECK("conv_bwd");
  return MACE_OK;
}

namespace {
// d up[n] = sum of the sender-side terms of the edges whose sender is n: the
// conv backward stores the term of edge x in the row of its reverse edge, so
// these are the contiguous rows of n's incoming edges.  A thread owns four
// consecutive features (16-byte loads) and keeps eight rows of loads in
// flight; eight partial sums over the rows in a fixed order (deterministic).
// With p.n_active, the rows whose term would come from an inactive receiver
// (the edge's sender is >= n_active) were never written and count as zero.
__global__ void k_dup_gather(ConvParams p) {
  const int64_t n = p.n0 + blockIdx.x;
  const int64_t e0 = p.row_ptr[n], e1 = p.row_ptr[n + 1];
  const int ne = (int)(e1 - e0);
  const int q4 = threadIdx.x;  // features 4 q4 .. 4 q4 + 3
  if (4 * q4 >= p.in_dim) return;
  const int64_t pitch = p.in_dim / 4;
  const float4* rows = reinterpret_cast<const float4*>(p.tq + e0 * p.in_dim) + q4;
  float4 acc[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) acc[b] = make_float4(0.f, 0.f, 0.f, 0.f);
  auto add = [](float4& a, const float4& v) {
    a.x += v.x;
    a.y += v.y;
    a.z += v.z;
    a.w += v.w;
  };
  const int32_t* snd = p.snd + e0;
  const int64_t na = p.n_active;
  auto live = [&](int jj) { return na == 0 || __ldg(snd + jj) < na; };
  const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
  int j = 0;
  for (; j + 8 <= ne; j += 8) {
    float4 v[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) v[b] = live(j + b) ? __ldg(rows + (j + b) * pitch) : zero;
#pragma unroll
    for (int b = 0; b < 8; ++b) add(acc[b], v[b]);
  }
#pragma unroll
  for (int b = 0; b < 8; ++b)
    if (j + b < ne && live(j + b)) add(acc[b], __ldg(rows + (j + b) * pitch));
#pragma unroll
  for (int b = 1; b < 8; b += 2) add(acc[b - 1], acc[b]);
  add(acc[0], acc[2]);
  add(acc[4], acc[6]);
  add(acc[0], acc[4]);
  reinterpret_cast<float4*>(p.dup + n * p.in_dim)[q4] = acc[0];
}
}  // namespace

int launch_dup_gather(const ConvParams& p, cudaStream_t s) {
  if (p.N <= p.n0) return MACE_OK;
  if (p.in_dim % 4 != 0 || p.in_dim > 4096) return fail(MACE_ERR_UNSUPPORTED, "dup_gather: input feature count");
  const int threads = (p.in_dim / 4 + 31) / 32 * 32;  // four features per thread
  k_dup_gather<<<(unsigned)(p.N - p.n0), threads, 0, s>>>(p);
  MACE_LAUNCH_CHECK("dup_gather");
  return MACE_OK;
}

}  // namespace mace
