// Interaction conv_tp + receiver-segmented sum, specialised per layer
// signature: the ordered list of (l1, l2, l3) paths of a layer and the channel
// count C are template parameters, so the path loop is unrolled at compile
// time and every per-path offset, table pitch and loop bound is a constant.
//
// Same mathematics and CTA layout as conv.cu (reference: conv_tp + scatter_sum
// in blocks.py:242-279, uvu semantics of tensor_product.py:833-1043); what the
// specialisation changes is the instruction count per (edge, channel):
//   * the sender's input features are loaded once per edge and shared by every
//     path with the same l1 (the generic kernel reloads them per path);
//   * the edge's spherical harmonics are held in registers for all paths;
//   * the per-edge M_k = CG.Y blocks and the per-receiver H tables are stored
//     flattened, padded to 4 floats, and read with 128-bit shared-memory loads;
//   * the radial weight of path k sits at a constant stride from path 0 in the
//     128-edge tile layout, so its address is formed once per edge;
//   * the backward's sender-side sums through the reverse edge accumulate in
//     registers (input slots 0e, 1o, 2e in that order, each C channels) and
//     reach shared memory once per receiver.
// Layers whose signature is not instantiated here use conv.cu.
#include <utility>

#include "common.cuh"

namespace mace {

namespace {

constexpr unsigned FULLMASK = 0xffffffffu;

__host__ __device__ constexpr int cl1(int code) { return code >> 4; }
__host__ __device__ constexpr int cl2(int code) { return (code >> 2) & 3; }
__host__ __device__ constexpr int cl3(int code) { return code & 3; }
__host__ __device__ constexpr int dim(int l) { return 2 * l + 1; }
__host__ __device__ constexpr int up4(int x) { return (x + 3) & ~3; }

// path code = l1 * 16 + l2 * 4 + l3
template <int... Codes>
struct Sig {
  static constexpr int n = sizeof...(Codes);
  __host__ __device__ static constexpr int code(int k) {
    constexpr int c[] = {Codes...};
    return c[k];
  }
  // H table (backward): per channel, per path the D1 x D2 block flattened and
  // padded to a multiple of 4 floats
  __host__ __device__ static constexpr int hoff(int k) {
    int s = 0;
    for (int i = 0; i < k; ++i) s += up4(dim(cl1(code(i))) * dim(cl2(code(i))));
    return s;
  }
  // pitch of a channel's H row: = 4 (mod 8) floats, so 8 lanes' 128-bit loads hit distinct banks
  __host__ __device__ static constexpr int hpitch() { return (hoff(n) % 8 == 0) ? hoff(n) + 4 : hoff(n); }
  // M rows (per edge): per path the D1 x D3 block flattened and padded to a
  // multiple of 4 floats
  __host__ __device__ static constexpr int moff(int k) {
    int s = 0;
    for (int i = 0; i < k; ++i) s += up4(dim(cl1(code(i))) * dim(cl3(code(i))));
    return s;
  }
  __host__ __device__ static constexpr int mtot() { return moff(n); }
  // forward accumulators: per path D3 values
  __host__ __device__ static constexpr int aoff(int k) {
    int s = 0;
    for (int i = 0; i < k; ++i) s += dim(cl3(code(i)));
    return s;
  }
  __host__ __device__ static constexpr int atot() { return aoff(n); }
  __host__ __device__ static constexpr int maxl1() {
    int m = 0;
    for (int i = 0; i < n; ++i) m = cl1(code(i)) > m ? cl1(code(i)) : m;
    return m;
  }
  __host__ __device__ static constexpr int in_ch() { return (maxl1() + 1) * (maxl1() + 1); }
};

template <class S, int... Ks, class F>
__device__ __forceinline__ void for_paths(std::integer_sequence<int, Ks...>, F&& f) {
  (f(std::integral_constant<int, Ks>{}), ...);
}
template <class S, class F>
__device__ __forceinline__ void each_path(F&& f) {
  for_paths<S>(std::make_integer_sequence<int, S::n>{}, f);
}

// Stage the senders, SH rows and (WITH_M) padded M rows of `ne` edges starting at cb.
template <class S, int EC, int NT, bool WITH_M = true>
__device__ __forceinline__ void stage(const ConvParams& p, int64_t cb, int ne, int* sSnd, float* sY, float* sM) {
  const int tid = threadIdx.x;
  for (int j = tid; j < ne; j += NT) sSnd[j] = p.snd[cb + j];
  for (int q = tid; q < ne * 16; q += NT) sY[q] = p.Y[cb * 16 + q];
  __syncthreads();
  if (!WITH_M) return;
  constexpr int MT = S::mtot();
  each_path<S>([&](auto kc) {
    constexpr int K = decltype(kc)::value;
    constexpr int CODE = S::code(K);
    constexpr int D1 = dim(cl1(CODE)), D2 = dim(cl2(CODE)), D3 = dim(cl3(CODE));
    constexpr int YO = cl2(CODE) * cl2(CODE), BLK = up4(D1 * D3), MO = S::moff(K);
    const float* cg = p.slot[K].cg;
    for (int idx = tid; idx < ne * BLK; idx += NT) {
      const int j = idx / BLK, r = idx - j * BLK;
      const int i = r / D3, m = r - i * D3;
      float acc = 0.f;
      if (r < D1 * D3) {
        const float* y = sY + j * 16 + YO;
#pragma unroll
        for (int jj = 0; jj < D2; ++jj) acc = fmaf(__ldg(cg + (i * D2 + jj) * D3 + m), y[jj], acc);
      }
      sM[j * MT + MO + r] = acc;
    }
  });
  __syncthreads();
}

// x[l1^2 + i] = up[s][slot l1][i][u] for the input slots 0e, 1o, 2e used
template <class S, int C>
__device__ __forceinline__ void load_sender(const ConvParams& p, int64_t s, int u, float* x) {
  const float* row = p.up + s * p.in_dim + u;
#pragma unroll
  for (int q = 0; q < S::in_ch(); ++q) x[q] = __ldg(row + q * C);
}

// ---------------------------------------------------------------------------
// forward: A[n][k][m][u] = sum_e w_e[k][u] sum_i x1[s_e][u][i] M_k,e[i][m]
// ---------------------------------------------------------------------------
template <int C, class S>
__global__ void __launch_bounds__(C) k_conv_fwd_sig(ConvParams p) {
  constexpr int EC = 64;
  constexpr int MT = S::mtot();
  extern __shared__ __align__(16) float sm[];
  int* sSnd = reinterpret_cast<int*>(sm);
  float* sY = sm + EC;
  float* sM = sY + EC * 16;
  const int64_t n = p.n0 + blockIdx.x;
  if (conv_receiver_skipped(p, n)) return;  // the other part of a split launch
  const int u = threadIdx.x;
  const int64_t e_beg = p.row_ptr[n], e_end = p.row_ptr[n + 1];
  float acc[S::atot()];
#pragma unroll
  for (int q = 0; q < S::atot(); ++q) acc[q] = 0.f;
  const int nch = p.wnch;
  constexpr int64_t KSTRIDE = (int64_t)(C / 32) * WT_CHUNK;  // path k+1 is this far from path k
  // EPI edges per step; the next EPI edges' sender features and radial
  // weights are loaded while these are computed (small signatures stream more
  // edges at once: their per-edge arithmetic is short)
  constexpr int EPI = S::n <= 4 ? 4 : (S::n <= 10 ? 2 : 1);
  float xn[EPI][S::in_ch()], wn[EPI][S::n];
  auto fetch = [&](int64_t cb, int j0, int ne) {
#pragma unroll
    for (int b = 0; b < EPI; ++b) {
      if (j0 + b >= ne) break;
      load_sender<S, C>(p, sSnd[j0 + b], u, xn[b]);
      const float* wp = p.w + wt_index(cb + j0 + b - p.e0, u, nch);
#pragma unroll
      for (int k = 0; k < S::n; ++k) wn[b][k] = __ldg(wp + k * KSTRIDE);
    }
  };
  for (int64_t cb = e_beg; cb < e_end; cb += EC) {
    const int ne = (int)imin64(EC, e_end - cb);
    stage<S, EC, C>(p, cb, ne, sSnd, sY, sM);
    fetch(cb, 0, ne);
    for (int j0 = 0; j0 < ne; j0 += EPI) {
      float xb[EPI][S::in_ch()], wb[EPI][S::n];
#pragma unroll
      for (int b = 0; b < EPI; ++b) {
#pragma unroll
        for (int q = 0; q < S::in_ch(); ++q) xb[b][q] = xn[b][q];
#pragma unroll
        for (int k = 0; k < S::n; ++k) wb[b][k] = wn[b][k];
      }
      if (j0 + EPI < ne) fetch(cb, j0 + EPI, ne);
#pragma unroll
      for (int b = 0; b < EPI; ++b) {
      const int j = j0 + b;
      if (j >= ne) break;
      const float* x = xb[b];
      const float* wv = wb[b];
      const float* Mrow = sM + j * MT;
      each_path<S>([&](auto kc) {
        constexpr int K = decltype(kc)::value;
        constexpr int CODE = S::code(K);
        constexpr int L1 = cl1(CODE), D1 = dim(L1), D3 = dim(cl3(CODE)), NQ = up4(D1 * D3) / 4;
        constexpr int XO = L1 * L1, AO = S::aoff(K);
        const float w = wv[K];
        const float4* mk = reinterpret_cast<const float4*>(Mrow + S::moff(K));
        float t[D3];
#pragma unroll
        for (int m = 0; m < D3; ++m) t[m] = 0.f;
        // flattened M block: entry f = i * D3 + m
#pragma unroll
        for (int q = 0; q < NQ; ++q) {
          const float4 v4 = mk[q];
          const float v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (4 * q + c < D1 * D3) t[(4 * q + c) % D3] = fmaf(x[XO + (4 * q + c) / D3], v[c], t[(4 * q + c) % D3]);
        }
#pragma unroll
        for (int m = 0; m < D3; ++m) acc[AO + m] = fmaf(w, t[m], acc[AO + m]);
      });
      }
    }
    __syncthreads();
  }
  float* out = p.A + n * p.mid_dim + u;
  each_path<S>([&](auto kc) {
    constexpr int K = decltype(kc)::value;
    constexpr int D3 = dim(cl3(S::code(K))), AO = S::aoff(K);
    const int off = p.slot[K].off;
#pragma unroll
    for (int m = 0; m < D3; ++m) out[off + m * C] = acc[AO + m];
  });
}

// ---------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------

// Sum 16 per-lane values over the warp; lane L ends with the total of index L>>1.
__device__ __forceinline__ float warp_sum16(float s[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const bool hi = lane & 16;
    const float keep = hi ? s[8 + i] : s[i];
    const float send = hi ? s[i] : s[8 + i];
    s[i] = keep + __shfl_xor_sync(FULLMASK, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const bool hi = lane & 8;
    const float keep = hi ? s[4 + i] : s[i];
    const float send = hi ? s[i] : s[4 + i];
    s[i] = keep + __shfl_xor_sync(FULLMASK, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const bool hi = lane & 4;
    const float keep = hi ? s[2 + i] : s[i];
    const float send = hi ? s[i] : s[2 + i];
    s[i] = keep + __shfl_xor_sync(FULLMASK, send, 4);
  }
  {
    const bool hi = lane & 2;
    const float keep = hi ? s[1] : s[0];
    const float send = hi ? s[0] : s[1];
    s[0] = keep + __shfl_xor_sync(FULLMASK, send, 2);
  }
  return s[0] + __shfl_xor_sync(FULLMASK, s[0], 1);
}

// MODE 0: no input gradient (first layer); 1: sender-side term gathered from
// the neighbours' dA (as conv.cu); 2: per-edge sender-side terms from this
// receiver's H tables, written to p.tq and summed by launch_dup_gather
template <int C, int G, class S, int MODE>
struct BwdLayout {
  static constexpr int EC = 32;
  static constexpr int NW = C / 32;  // warps per group
  static constexpr int HP = S::hpitch();
  static constexpr int SND = 0;
  static constexpr int Y = SND + EC;
  static constexpr int M = Y + EC * 16;
  static constexpr int RED = M + (MODE == 1 ? EC * S::mtot() : 0);
  static constexpr int H = RED + NW * EC * 16;
  static constexpr int DUP = H + C * HP;
  static constexpr int TOTAL = DUP + (MODE == 1 ? G * S::in_ch() * C : 0);  // floats
};

// Per receiver n, path k and channel u the receiver's gradient enters every
// edge only through H_k[i][j] = sum_m pw CG_k[i, j, m] dA[n][k][m][u], built
// once per CTA; then per edge
//   dw_e[k, u] = sum_{i,j} x1[i] H[i][j] Y_e[j],   dY_e[j] += w sum_i x1[i] H[i][j],
// and the gradient of the sender's features, either (MODE 1) gathered at the
// sender's own CTA through the reverse edge,
//   d up[n][l1 slot][i][u] += (-1)^l2 w sum_m M_k,e[i][m] dA[s_e][k][m][u],
// or (MODE 2) formed here from the same H block and written per edge into
// the row of its reverse edge,
//   T_e[l1 slot][i][u] = sum_k w_e[k, u] sum_j H_k[i][j] Y_e[j]  -> tq[rev(e)],
// for launch_dup_gather to sum over each node's (contiguous) incoming rows.
// G groups of C threads share one receiver: group g takes edges g, g+G, ...
// Three CTAs per SM (at most 85 registers a thread at 256 threads) where the
// signature has at most 10 paths: the medium model's layers then compile
// without spills and the extra warps hide the sender and weight loads.
template <int C, int G, class S, int MODE>
__global__ void __launch_bounds__(C * G, (S::n <= 10 ? 3 : 2)) k_conv_bwd_sig(ConvParams p) {
  using Lay = BwdLayout<C, G, S, MODE>;
  constexpr int EC = Lay::EC, NW = Lay::NW, HP = Lay::HP, MT = S::mtot(), IC = S::in_ch();
  constexpr int NT = C * G;
  extern __shared__ __align__(16) float sm[];
  int* sSnd = reinterpret_cast<int*>(sm + Lay::SND);
  float* sY = sm + Lay::Y;
  float* sM = sm + Lay::M;
  float* sRed = sm + Lay::RED;
  float* sH = sm + Lay::H;
  float* sDup = sm + Lay::DUP;
  const int64_t n = p.n0 + blockIdx.x;
  if (conv_receiver_skipped(p, n)) return;  // the other part of a split launch
  const int tid = threadIdx.x;
  const int u = tid % C, grp = tid / C;
  const int warp = u >> 5, lane = tid & 31;
  const int64_t e_beg = p.row_ptr[n], e_end = p.row_ptr[n + 1];
  // H tables, paths split over the groups
  {
    const float* g = p.dA + n * p.mid_dim + u;
    each_path<S>([&](auto kc) {
      constexpr int K = decltype(kc)::value;
      constexpr int CODE = S::code(K);
      constexpr int D1 = dim(cl1(CODE)), D2 = dim(cl2(CODE)), D3 = dim(cl3(CODE));
      if (K % G != grp) return;
      const ConvSlotDev& sl = p.slot[K];
      float gk[D3];
#pragma unroll
      for (int m = 0; m < D3; ++m) gk[m] = g[sl.off + m * C];
      float* h = sH + u * HP + S::hoff(K);
      // flattened block: entry f = i * D2 + j
#pragma unroll
      for (int f = 0; f < up4(D1 * D2); ++f) {
        float a = 0.f;
        if (f < D1 * D2) {
#pragma unroll
          for (int m = 0; m < D3; ++m) a = fmaf(__ldg(sl.cg + f * D3 + m), gk[m], a);
        }
        h[f] = a;
      }
    });
  }
  __syncthreads();
  float dup[MODE == 1 ? IC : 1];
#pragma unroll
  for (int q = 0; q < (MODE == 1 ? IC : 1); ++q) dup[q] = 0.f;
  const int nch = p.wnch;
  constexpr int64_t KSTRIDE = (int64_t)(C / 32) * WT_CHUNK;
  const float4* hrow = reinterpret_cast<const float4*>(sH + u * HP);
  // EPI of this group's edges per step; the next EPI edges' sender features
  // and radial weights are loaded while these are computed
  constexpr int EPI = S::n <= 4 ? 4 : 1;
  float xn[EPI][IC], wn[EPI][S::n];
  auto fetch = [&](int64_t cb, int j0, int ne) {
#pragma unroll
    for (int b = 0; b < EPI; ++b) {
      const int j = j0 + b * G;
      if (j >= ne) break;
      load_sender<S, C>(p, sSnd[j], u, xn[b]);
      const float* wp = p.w + wt_index(cb + j - p.e0, u, nch);
#pragma unroll
      for (int k = 0; k < S::n; ++k) wn[b][k] = __ldg(wp + k * KSTRIDE);
    }
  };
  for (int64_t cb = e_beg; cb < e_end; cb += EC) {
    const int ne = (int)imin64(EC, e_end - cb);
    stage<S, EC, NT, MODE == 1>(p, cb, ne, sSnd, sY, sM);
    fetch(cb, grp, ne);
    for (int j0 = grp; j0 < ne; j0 += EPI * G) {
      float xb[EPI][IC], wb[EPI][S::n];
#pragma unroll
      for (int b = 0; b < EPI; ++b) {
#pragma unroll
        for (int q = 0; q < IC; ++q) xb[b][q] = xn[b][q];
#pragma unroll
        for (int k = 0; k < S::n; ++k) wb[b][k] = wn[b][k];
      }
      if (j0 + EPI * G < ne) fetch(cb, j0 + EPI * G, ne);
#pragma unroll
      for (int b = 0; b < EPI; ++b) {
      const int j = j0 + b * G;
      if (j >= ne) break;
      const int64_t e = cb + j;
      const int64_t s = sSnd[j];
      float tq[MODE == 2 ? IC : 1];
#pragma unroll
      for (int q = 0; q < (MODE == 2 ? IC : 1); ++q) tq[q] = 0.f;
      float Ye[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 v = reinterpret_cast<const float4*>(sY + j * 16)[q];
        Ye[4 * q] = v.x;
        Ye[4 * q + 1] = v.y;
        Ye[4 * q + 2] = v.z;
        Ye[4 * q + 3] = v.w;
      }
      const float* x = xb[b];
      const float* wv = wb[b];
      const int64_t wi = wt_index(e - p.e0, u, nch);
      float* dwp = p.dw + wi;
      const float* dAs = p.dA + s * p.mid_dim + u;
      const float4* mrow = reinterpret_cast<const float4*>(sM + j * MT);
      float sdy[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) sdy[q] = 0.f;
      each_path<S>([&](auto kc) {
        constexpr int K = decltype(kc)::value;
        constexpr int CODE = S::code(K);
        constexpr int L1 = cl1(CODE), L2 = cl2(CODE);
        constexpr int D1 = dim(L1), D2 = dim(L2), D3 = dim(cl3(CODE));
        constexpr int HQ = up4(D1 * D2) / 4, MQ = up4(D1 * D3) / 4;
        constexpr int XO = L1 * L1, YO = L2 * L2;
        constexpr float PAR = (L2 & 1) ? -1.f : 1.f;
        const float w = wv[K];
        // xh[j] = sum_i x1[i] H[i][j]; th[i] = sum_j H[i][j] Y[j]   (flattened H block: f = i * D2 + j)
        float xh[D2], th[D1];
#pragma unroll
        for (int jj = 0; jj < D2; ++jj) xh[jj] = 0.f;
#pragma unroll
        for (int i = 0; i < D1; ++i) th[i] = 0.f;
#pragma unroll
        for (int q = 0; q < HQ; ++q) {
          const float4 h4 = hrow[S::hoff(K) / 4 + q];
          const float h[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
          for (int c = 0; c < 4; ++c)
            if (4 * q + c < D1 * D2) {
              const int i = (4 * q + c) / D2, jj = (4 * q + c) % D2;
              xh[jj] = fmaf(x[XO + i], h[c], xh[jj]);
              if (MODE == 2) th[i] = fmaf(h[c], Ye[YO + jj], th[i]);
            }
        }
        if constexpr (MODE == 2) {
#pragma unroll
          for (int i = 0; i < D1; ++i) tq[XO + i] = fmaf(w, th[i], tq[XO + i]);
        }
        float dw = 0.f;
#pragma unroll
        for (int jj = 0; jj < D2; ++jj) {
          dw = fmaf(xh[jj], Ye[YO + jj], dw);
          sdy[YO + jj] = fmaf(w, xh[jj], sdy[YO + jj]);
        }
        dwp[K * KSTRIDE] = dw;
        if constexpr (MODE == 1) {
          // sender side through the reverse edge: r[i] = sum_m M[i][m] gr[m]   (f = i * D3 + m)
          const int off = p.slot[K].off;
          float gr[D3];
#pragma unroll
          for (int m = 0; m < D3; ++m) gr[m] = __ldg(dAs + off + m * C);
          float r[D1];
#pragma unroll
          for (int i = 0; i < D1; ++i) r[i] = 0.f;
#pragma unroll
          for (int q = 0; q < MQ; ++q) {
            const float4 m4 = mrow[S::moff(K) / 4 + q];
            const float mv[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
            for (int c = 0; c < 4; ++c)
              if (4 * q + c < D1 * D3) r[(4 * q + c) / D3] = fmaf(mv[c], gr[(4 * q + c) % D3], r[(4 * q + c) / D3]);
          }
#pragma unroll
          for (int i = 0; i < D1; ++i) dup[XO + i] = fmaf(PAR * w, r[i], dup[XO + i]);
        }
      });
      if constexpr (MODE == 2) {
        // stored at the reverse edge's row: a node's terms are then the
        // contiguous rows of its own incoming edges
        float* tp = p.tq + (int64_t)__ldg(p.rev + e) * (IC * C) + u;
#pragma unroll
        for (int q = 0; q < IC; ++q) tp[q * C] = tq[q];
      }
      const float tot = warp_sum16(sdy);
      if ((lane & 1) == 0) sRed[(warp * EC + j) * 16 + (lane >> 1)] = tot;
      }
    }
    __syncthreads();
    for (int idx = tid; idx < ne * 16; idx += NT) {
      const int j = idx >> 4, q = idx & 15;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < NW; ++w) v += sRed[(w * EC + j) * 16 + q];
      p.dY[(cb + j) * 16 + q] += v;
    }
    __syncthreads();
  }
  if constexpr (MODE == 1) {
#pragma unroll
    for (int q = 0; q < IC; ++q) sDup[(grp * IC + q) * C + u] = dup[q];
    __syncthreads();
    for (int q = tid; q < IC * C; q += NT) {
      float v = 0.f;
#pragma unroll
      for (int g = 0; g < G; ++g) v += sDup[g * IC * C + q];  // fixed order: deterministic
      p.dup[n * p.in_dim + q] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// dispatch
// ---------------------------------------------------------------------------
template <class S>
bool sig_matches(const ConvParams& p) {
  if (p.n_mid != S::n || p.in_dim != S::in_ch() * p.C) return false;
  for (int k = 0; k < S::n; ++k) {
    const ConvSlotDev& sl = p.slot[k];
    const int code = S::code(k);
    if (sl.l1 != cl1(code) || sl.l2 != cl2(code) || sl.l3 != cl3(code)) return false;
    if (sl.src_ch != sl.l1 * sl.l1 || sl.src_off != sl.l1 * sl.l1 * p.C) return false;
  }
  return true;
}

template <int C, class S>
int run_fwd(const ConvParams& p, cudaStream_t s) {
  const size_t smem = (size_t)(64 + 64 * 16 + 64 * S::mtot()) * sizeof(float);
  MACE_CUDA_TRY(cudaFuncSetAttribute(k_conv_fwd_sig<C, S>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_conv_fwd_sig<C, S><<<(unsigned)(p.N - p.n0), C, smem, s>>>(p);
  MACE_LAUNCH_CHECK("conv_fwd_sig");
  return MACE_OK;
}

template <int C, int G, class S, int MODE>
int run_bwd_mode(const ConvParams& p, cudaStream_t s) {
  const size_t smem = (size_t)BwdLayout<C, G, S, MODE>::TOTAL * sizeof(float);
  if (smem > 227 * 1024) return fail(MACE_ERR_UNSUPPORTED, "conv backward tile exceeds shared memory");
  MACE_CUDA_TRY(
      cudaFuncSetAttribute(k_conv_bwd_sig<C, G, S, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_conv_bwd_sig<C, G, S, MODE><<<(unsigned)(p.N - p.n0), C * G, smem, s>>>(p);
  MACE_LAUNCH_CHECK("conv_bwd_sig");
  return MACE_OK;
}

template <int C, int G, class S>
int run_bwd(const ConvParams& p, cudaStream_t s, bool* need_gather) {
  *need_gather = false;
  if (!p.need_dup) return run_bwd_mode<C, G, S, 0>(p, s);
  if (p.tq && p.in_dim == S::in_ch() * C) {
    *need_gather = true;
    return run_bwd_mode<C, G, S, 2>(p, s);
  }
  return run_bwd_mode<C, G, S, 1>(p, s);
}

// layer signatures of the MACE families in use: input 0e only (first layer,
// and every layer of 0e-only models), 0e+1o inputs (max_L = 1), 0e+1o+2e
// inputs (max_L = 2), each with SH up to l = 3
using SigL0 = Sig<0x00, 0x05, 0x0A, 0x0F>;
using SigL1 = Sig<0x00, 0x14, 0x05, 0x11, 0x19, 0x0A, 0x16, 0x1E, 0x0F, 0x1B>;
using SigL2 = Sig<0x00, 0x14, 0x28, 0x05, 0x11, 0x19, 0x25, 0x2D, 0x0A, 0x16, 0x1E, 0x22, 0x2A, 0x0F, 0x1B,
                  0x27, 0x2F>;

template <int C>
int try_fwd(const ConvParams& p, cudaStream_t s, bool* used) {
  *used = true;
  if (sig_matches<SigL0>(p)) return run_fwd<C, SigL0>(p, s);
  if (sig_matches<SigL1>(p)) return run_fwd<C, SigL1>(p, s);
  if (sig_matches<SigL2>(p)) return run_fwd<C, SigL2>(p, s);
  *used = false;
  return MACE_OK;
}

template <int C>
int try_bwd(const ConvParams& p, cudaStream_t s, bool* used, bool* need_gather) {
  *used = true;
  if (sig_matches<SigL0>(p)) return run_bwd<C, 2, SigL0>(p, s, need_gather);
  if (sig_matches<SigL1>(p)) return run_bwd<C, 2, SigL1>(p, s, need_gather);
  if (sig_matches<SigL2>(p)) return run_bwd<C, 2, SigL2>(p, s, need_gather);
  *used = false;
  return MACE_OK;
}

}  // namespace

int launch_conv_fwd_sig(const ConvParams& p, cudaStream_t s, bool* used) {
  *used = false;
  if (p.C == 128) return try_fwd<128>(p, s, used);
  if (p.C == 96) return try_fwd<96>(p, s, used);
  return MACE_OK;
}

int launch_conv_bwd_sig(const ConvParams& p, cudaStream_t s, bool* used, bool* need_gather) {
  *used = false;
  *need_gather = false;
  if (p.C == 128) return try_bwd<128>(p, s, used, need_gather);
  if (p.C == 96) return try_bwd<96>(p, s, used, need_gather);
  return MACE_OK;
}

}  // namespace mace
