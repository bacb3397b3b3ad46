// Per-receiver sums of the mpa-0 family's element- and length-dependent
// terms, and the density normalisation of the interaction message.
//
// Reference semantics:
//   density: d_e = tanh((w_d . b_e)^2), D_n = sum_{e -> n} d_e,
//            message_n = linear(A)_n / (D_n + 1)        (mace_mlx/blocks.py:389-401)
//   ZBL:     E_pair,n = sum_{e -> n} 0.5 * 14.3996 Z_s Z_r / r_e * phi(r_e / a)
//                                   * envelope_p(r_e / (R_s + R_r))
//                                                       (mace_mlx/radial.py:160-197)
// One warp per receiver walks its CSR row (edges are sorted by receiver) and a
// fixed shuffle tree sums the lanes, so the sums are deterministic.  The
// gradients of both terms with respect to the edge lengths are formed in the
// edge backward kernel (edge.cu) from the per-receiver seeds computed here.
#include "common.cuh"

namespace mace {

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void k_node_sums(NodeSumParams p) {
  const int64_t n = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= p.N) return;
  const int e0 = p.row_ptr[n], e1 = p.row_ptr[n + 1];
  float dsum[MACE_MAX_LAYERS] = {0.f, 0.f, 0.f, 0.f};
  float pair = 0.f;
  const int zr = p.species[n];
  for (int e = e0 + lane; e < e1; e += 32) {
    const float* b = p.b + (int64_t)e * p.nb;
    for (int t = 0; t < p.n_dens; ++t) {
      const float* wd = p.dens_w[t];
      float x = 0.f;
      for (int k = 0; k < p.nb; ++k) x = fmaf(__ldg(wd + k), b[k], x);
      dsum[t] += tanhf(x * x);
    }
    if (p.zbl) {
      const float v0 = p.v[3 * (int64_t)e], v1 = p.v[3 * (int64_t)e + 1], v2 = p.v[3 * (int64_t)e + 2];
      const float sq = __fadd_rn(__fadd_rn(__fmul_rn(v0, v0), __fmul_rn(v1, v1)), __fmul_rn(v2, v2));
      const float r = sqrtf(fmaxf(sq, 1e-24f));
      const int zs = p.species[p.snd[e]];
      float dvdr;
      pair += zbl_pair(r, __ldg(p.znum + zs), __ldg(p.znum + zr), __ldg(p.zbl_radius + zs) + __ldg(p.zbl_radius + zr),
                       p.zbl_a_exp, p.zbl_a_pref, p.zbl_p, &dvdr);
    }
  }
  for (int t = 0; t < p.n_dens; ++t) {
    const float d = warp_sum(dsum[t]);
    if (lane == 0) p.D[t][n] = d;
  }
  if (p.zbl) {
    pair = warp_sum(pair);
    if (lane == 0) p.pair[n] = pair;
  }
}

__global__ void k_density_scale(float* rows, int64_t row_len, const float* D, int64_t total) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= total) return;
  rows[i] = rows[i] / (D[i / row_len] + 1.0f);
}

// warp per node: dD = -(drows . rows) / (D + 1), drows /= (D + 1)
__global__ void k_density_bwd(const float* rows, float* drows, int64_t row_len, const float* D, float* dD,
                              int64_t N) {
  const int64_t n = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const float* r = rows + n * row_len;
  float* g = drows + n * row_len;
  const float den = D[n] + 1.0f;
  float acc = 0.f;
  for (int64_t f = lane; f < row_len; f += 32) {
    const float gv = g[f];
    acc = fmaf(gv, r[f], acc);
    g[f] = gv / den;
  }
  acc = warp_sum(acc);
  if (lane == 0) dD[n] = -acc / den;
}

}  // namespace

int launch_node_sums(const NodeSumParams& p, cudaStream_t s) {
  if (p.N == 0 || (p.n_dens == 0 && !p.zbl)) return MACE_OK;
  if (p.n_dens > MACE_MAX_LAYERS) return fail(MACE_ERR_UNSUPPORTED, "node sums: too many density layers");
  k_node_sums<<<(unsigned)((p.N * 32 + 255) / 256), 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("node_sums");
  return MACE_OK;
}

int launch_density_scale(float* rows, int64_t row_len, const float* D, int64_t N, cudaStream_t s) {
  const int64_t total = N * row_len;
  if (total == 0) return MACE_OK;
  k_density_scale<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(rows, row_len, D, total);
  MACE_LAUNCH_CHECK("density_scale");
  return MACE_OK;
}

int launch_density_bwd(const float* rows, float* drows, int64_t row_len, const float* D, float* dD, int64_t N,
                       cudaStream_t s) {
  if (N == 0) return MACE_OK;
  k_density_bwd<<<(unsigned)((N * 32 + 255) / 256), 256, 0, s>>>(rows, drows, row_len, D, dD, N);
  MACE_LAUNCH_CHECK("density_bwd");
  return MACE_OK;
}

}  // namespace mace
