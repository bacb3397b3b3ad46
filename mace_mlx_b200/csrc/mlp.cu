// Radial MLP of the interaction blocks: bias-free Linear layers with SiLU in
// between, last layer without activation (mace_mlx/radial.py:329-341; the
// e3nn normalisation is already folded into the converted weights).
// Input: per-edge radial features b (E, nb); output: per-edge tensor-product
// weights (E, W).  The backward returns dL/db given dL/dW (input gradients
// only; weight gradients are never needed for forces).
//
// Layout: CTA of 256 threads owns a tile of TE = 32 edges.  Hidden
// activations live in shared memory; the wide last layer keeps one weight
// column chunk per thread in registers and streams edges from shared memory.
#include "common.cuh"

namespace mace {

namespace {

constexpr int TE = 32;
constexpr int NT = 256;

// dense layer on a shared-memory tile: out[e][o] = sum_i in[e][i] * W[i][o]
__device__ __forceinline__ void tile_layer(const float* __restrict__ W, int din, int dout,
                                           const float* sin, int ldin, float* sout, int ldout,
                                           int ne) {
  for (int idx = threadIdx.x; idx < TE * dout; idx += NT) {
    int e = idx / dout, o = idx % dout;
    float acc = 0.f;
    if (e < ne) {
      const float* x = sin + e * ldin;
      for (int i = 0; i < din; ++i) acc = fmaf(x[i], __ldg(W + i * dout + o), acc);
    }
    sout[e * ldout + o] = acc;
  }
}

template <int H>
__global__ void __launch_bounds__(NT) k_mlp_fwd(MlpParams p) {
  extern __shared__ float sm[];
  const int ld = H;  // all tile reads are warp-broadcasts: no padding needed
  float* s0 = sm;            // TE x ld
  float* s1 = sm + TE * ld;  // TE x ld
  const int64_t e0 = (int64_t)blockIdx.x * TE;
  const int ne = (int)imin64(TE, p.E - e0);
  const int nb = p.widths[0];
  const int nh = p.n_layers - 1;  // hidden layers
  const int wout = p.widths[p.n_layers];
  // stage the radial features
  for (int idx = threadIdx.x; idx < TE * nb; idx += NT) {
    int e = idx / nb, i = idx % nb;
    s0[e * ld + i] = (e < ne) ? p.b[(e0 + e) * nb + i] : 0.f;
  }
  __syncthreads();
  float* cur = s0;
  float* nxt = s1;
  for (int j = 0; j < nh; ++j) {
    const int din = p.widths[j];
    tile_layer(p.w[j], din, H, cur, ld, nxt, ld, ne);
    __syncthreads();
    for (int idx = threadIdx.x; idx < TE * H; idx += NT) {
      int e = idx / H, o = idx % H;
      float a = nxt[e * ld + o];
      if (e < ne) p.act[(e0 + e) * (int64_t)(nh * H) + j * H + o] = a;
      nxt[e * ld + o] = silu_f(a);
    }
    __syncthreads();
    float* t = cur;
    cur = nxt;
    nxt = t;
  }
  // last layer: H -> wout, one output column per thread per chunk
  const float* __restrict__ W = p.w[nh];
  for (int c0 = 0; c0 < wout; c0 += NT) {
    const int c = c0 + threadIdx.x;
    const bool ok = c < wout;
    float acc[TE];
#pragma unroll
    for (int e = 0; e < TE; ++e) acc[e] = 0.f;
#pragma unroll
    for (int i0 = 0; i0 < H; i0 += 16) {
      float wc[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) wc[i] = ok ? __ldg(W + (int64_t)(i0 + i) * wout + c) : 0.f;
#pragma unroll
      for (int e = 0; e < TE; ++e) {
        const float4* x4 = reinterpret_cast<const float4*>(cur + e * ld + i0);
        float a = acc[e];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float4 x = x4[q];
          a = fmaf(x.x, wc[4 * q + 0], a);
          a = fmaf(x.y, wc[4 * q + 1], a);
          a = fmaf(x.z, wc[4 * q + 2], a);
          a = fmaf(x.w, wc[4 * q + 3], a);
        }
        acc[e] = a;
      }
    }
    if (ok) {
#pragma unroll
      for (int e = 0; e < TE; ++e)
        if (e < ne) p.out[wt_index(e0 + e, c, wt_nchunk(wout))] = acc[e];
    }
  }
}

template <int H>
__global__ void __launch_bounds__(NT) k_mlp_bwd(MlpParams p) {
  extern __shared__ float sm[];
  constexpr int KC = 32;              // chunk of the wide dimension
  constexpr int IG = H / 4;           // groups of 4 hidden units
  constexpr int EG = NT / IG;         // edge groups
  constexpr int EPT = TE / EG;        // edges per thread
  static_assert(TE % EG == 0, "tile");
  const int ld = H + 1;
  float* sD = sm;                     // TE x (KC+1)   dout chunk
  float* sW = sD + TE * (KC + 1);     // KC x H        W^T chunk
  float* s0 = sW + KC * H;            // TE x ld
  float* s1 = s0 + TE * ld;           // TE x ld
  const int64_t e0 = (int64_t)blockIdx.x * TE;
  const int ne = (int)imin64(TE, p.E - e0);
  const int nh = p.n_layers - 1;
  const int wout = p.widths[p.n_layers];
  const float* __restrict__ Wt = p.wt[nh];  // (wout, H): the last layer's (out, in) matrix
  const int tig = threadIdx.x % IG, teg = threadIdx.x / IG;
  float acc[EPT][4];
#pragma unroll
  for (int a = 0; a < EPT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  for (int c0 = 0; c0 < wout; c0 += KC) {
    const int kc = min(KC, wout - c0);
    for (int idx = threadIdx.x; idx < TE * KC; idx += NT) {
      int e = idx / KC, c = idx % KC;
      sD[e * (KC + 1) + c] = (e < ne && c < kc) ? p.dout[wt_index(e0 + e, c0 + c, wt_nchunk(wout))] : 0.f;
    }
    for (int idx = threadIdx.x; idx < KC * H; idx += NT) {
      int c = idx / H, i = idx % H;
      sW[c * H + i] = (c < kc) ? __ldg(Wt + (int64_t)(c0 + c) * H + i) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < KC; ++c) {
      float4 w4 = *reinterpret_cast<const float4*>(sW + c * H + tig * 4);
#pragma unroll
      for (int a = 0; a < EPT; ++a) {
        float d = sD[(teg * EPT + a) * (KC + 1) + c];
        acc[a][0] = fmaf(d, w4.x, acc[a][0]);
        acc[a][1] = fmaf(d, w4.y, acc[a][1]);
        acc[a][2] = fmaf(d, w4.z, acc[a][2]);
        acc[a][3] = fmaf(d, w4.w, acc[a][3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < EPT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) s0[(teg * EPT + a) * ld + tig * 4 + b] = acc[a][b];
  __syncthreads();
  // back through the hidden layers: dh (s0) -> da = dh * silu'(a) -> dh_prev
  float* cur = s0;
  float* nxt = s1;
  for (int j = nh - 1; j >= 0; --j) {
    for (int idx = threadIdx.x; idx < TE * H; idx += NT) {
      int e = idx / H, o = idx % H;
      float a = (e < ne) ? p.act[(e0 + e) * (int64_t)(nh * H) + j * H + o] : 0.f;
      cur[e * ld + o] *= silu_grad_f(a);
    }
    __syncthreads();
    const int din = p.widths[j];
    // dh_prev[e][i] = sum_o da[e][o] * W_j[i][o]  == da @ W_j^T ; wt[j] is (H, din)
    tile_layer(p.wt[j], H, din, cur, ld, nxt, ld, ne);
    __syncthreads();
    float* t = cur;
    cur = nxt;
    nxt = t;
  }
  const int nb = p.widths[0];
  for (int idx = threadIdx.x; idx < TE * nb; idx += NT) {
    int e = idx / nb, i = idx % nb;
    if (e < ne) p.db[(e0 + e) * nb + i] += cur[e * ld + i];
  }
}

template <int H>
int mlp_fwd_h(const MlpParams& p, cudaStream_t s) {
  size_t smem = 2 * TE * H * sizeof(float);
  unsigned blocks = (unsigned)((p.E + TE - 1) / TE);
  k_mlp_fwd<H><<<blocks, NT, smem, s>>>(p);
  MACE_LAUNCH_CHECK("mlp_fwd");
  return MACE_OK;
}

template <int H>
int mlp_bwd_h(const MlpParams& p, cudaStream_t s) {
  size_t smem = (TE * 33 + 32 * H + 2 * TE * (H + 1)) * sizeof(float);
  if (smem > 48 * 1024) {
    cudaFuncSetAttribute(k_mlp_bwd<H>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  unsigned blocks = (unsigned)((p.E + TE - 1) / TE);
  k_mlp_bwd<H><<<blocks, NT, smem, s>>>(p);
  MACE_LAUNCH_CHECK("mlp_bwd");
  return MACE_OK;
}

int check_mlp(const MlpParams& p) {
  if (p.n_layers < 2 || p.n_layers > 7) return fail(MACE_ERR_UNSUPPORTED, "radial MLP needs 2..7 layers");
  int H = p.widths[1];
  for (int j = 1; j < p.n_layers; ++j)
    if (p.widths[j] != H) return fail(MACE_ERR_UNSUPPORTED, "radial MLP hidden widths must be equal");
  if (p.widths[0] > H) return fail(MACE_ERR_UNSUPPORTED, "radial MLP input wider than hidden");
  if (H != 32 && H != 64 && H != 128)
    return fail(MACE_ERR_UNSUPPORTED, "radial MLP hidden width must be 32, 64 or 128");
  return MACE_OK;
}

// apply_cutoff=False models (reference blocks.py:163-164, radial.py:313-317):
// the envelope multiplies the radial-MLP output, w_e = cut_e * MLP(b_e).  One
// warp per edge walks the edge's row of the tiled output (lane j takes the
// columns j, j + 32, ...; each 32-column step is one 128-byte line).
__global__ void k_cut_scale(float* out, const float* cut, int64_t E, int W, int nch) {
  const int64_t e = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (e >= E) return;
  const float c = cut[e];
  for (int k = lane; k < W; k += 32) out[wt_index(e, k, nch)] *= c;
}

// Backward of the scaling: dE/dcut_e = sum_k dw[e][k] * w_raw[e][k] with
// w_raw = w / cut_e (an edge whose envelope is 0 has dcut/dr = 0 as well, so
// it adds nothing), accumulated over layers into dcut; then dw[e] *= cut_e,
// the gradient the MLP backward takes.  Fixed shuffle tree: deterministic.
__global__ void k_cut_bwd(float* dout, const float* out, const float* cut, float* dcut, int64_t E, int W, int nch) {
  const int64_t e = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (e >= E) return;
  const float c = cut[e];
  float acc = 0.f;
  for (int k = lane; k < W; k += 32) {
    const int64_t i = wt_index(e, k, nch);
    const float g = dout[i];
    acc = fmaf(g, out[i], acc);
    dout[i] = g * c;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0 && c > 0.f) dcut[e] += acc / c;
}

int cut_scale(const MlpParams& p, cudaStream_t s) {
  const int W = p.widths[p.n_layers];
  k_cut_scale<<<(unsigned)((p.E * 32 + 255) / 256), 256, 0, s>>>(p.out, p.cut, p.E, W, wt_nchunk(W));
  MACE_LAUNCH_CHECK("mlp_cut_scale");
  return MACE_OK;
}

int cut_bwd(const MlpParams& p, cudaStream_t s) {
  const int W = p.widths[p.n_layers];
  k_cut_bwd<<<(unsigned)((p.E * 32 + 255) / 256), 256, 0, s>>>(const_cast<float*>(p.dout), p.out, p.cut, p.dcut,
                                                               p.E, W, wt_nchunk(W));
  MACE_LAUNCH_CHECK("mlp_cut_bwd");
  return MACE_OK;
}

int mlp_fwd_any(const MlpParams& p, cudaStream_t s) {
  if (mlp_tc_supported(p)) return launch_mlp_fwd_tc(p, s);
  int rc = check_mlp(p);
  if (rc) return rc;
  switch (p.widths[1]) {
    case 32: return mlp_fwd_h<32>(p, s);
    case 64: return mlp_fwd_h<64>(p, s);
    default: return mlp_fwd_h<128>(p, s);
  }
}

}  // namespace

int launch_mlp_fwd(const MlpParams& p, cudaStream_t s) {
  if (p.E == 0) return MACE_OK;
  int rc = mlp_fwd_any(p, s);
  if (rc || !p.cut) return rc;
  return cut_scale(p, s);
}

int launch_mlp_bwd(const MlpParams& p, cudaStream_t s) {
  if (p.E == 0) return MACE_OK;
  if (p.cut) {
    int rc = cut_bwd(p, s);
    if (rc) return rc;
  }
  if (mlp_tc_supported(p)) return launch_mlp_bwd_tc(p, s);
  int rc = check_mlp(p);
  if (rc) return rc;
  switch (p.widths[1]) {
    case 32: return mlp_bwd_h<32>(p, s);
    case 64: return mlp_bwd_h<64>(p, s);
    default: return mlp_bwd_h<128>(p, s);
  }
}

}  // namespace mace
