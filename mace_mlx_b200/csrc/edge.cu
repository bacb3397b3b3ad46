// Edge front end: geometry, spherical harmonics, Bessel basis x cutoff
// envelope (forward and hand-written backward), forces and virial assembly.
//
// Reference semantics:
//   v = pos[receiver] - pos[sender] + shifts @ cell, r = sqrt(max(|v|^2, 1e-24))
//                                          (mace_mlx/utils.py:47-84)
//   Y_0 = 1, Y_1 = sqrt(3) * v/r (e3nn seed), Y_l = T_l . (Y_{l-1} x Y_1)
//                                          (mace_mlx/spherical_harmonics.py:67-155)
//   b_n = sqrt(2/r_max) sin(w_n r)/r * envelope(r/r_max)
//                                          (mace_mlx/radial.py:18-71, 265-321)
//   with the Agnesi transform, the Bessel argument is r_t(r, element pair)
//   and the envelope keeps the raw r     (mace_mlx/radial.py:202-262, 294-321)
// The backward also carries the gradients of two element-dependent terms
// that depend on the edge length alone: the ZBL pair repulsion
// (radial.py:127-199) and the density normalisation's per-edge density
// tanh((w_d . b_e)^2) (blocks.py:389-401), whose per-receiver gradients the
// node kernels provide.
// One thread per edge; every edge's result is a pure function of its own
// inputs, so the reverse edge (j -> i, -S) gets bitwise v_rev = -v and the
// same r, which the conv backward relies on.
#include "common.cuh"

namespace mace {

namespace {

struct EdgeGeom {
  float v[3];
  float r;
  float u[3];
  bool clamped;
};

__device__ __forceinline__ EdgeGeom edge_geom(const EdgeParams& p, int64_t e) {
  EdgeGeom g;
  int s = p.snd[e], r = p.rcv[e];
  float v0 = p.pos[3 * r + 0] - p.pos[3 * s + 0];
  float v1 = p.pos[3 * r + 1] - p.pos[3 * s + 1];
  float v2 = p.pos[3 * r + 2] - p.pos[3 * s + 2];
  if (p.cell != nullptr) {
    float S0 = (float)p.shifts[3 * e + 0];
    float S1 = (float)p.shifts[3 * e + 1];
    float S2 = (float)p.shifts[3 * e + 2];
    const float* c = p.cell;
    float o0 = __fadd_rn(__fadd_rn(__fmul_rn(S0, c[0]), __fmul_rn(S1, c[3])), __fmul_rn(S2, c[6]));
    float o1 = __fadd_rn(__fadd_rn(__fmul_rn(S0, c[1]), __fmul_rn(S1, c[4])), __fmul_rn(S2, c[7]));
    float o2 = __fadd_rn(__fadd_rn(__fmul_rn(S0, c[2]), __fmul_rn(S1, c[5])), __fmul_rn(S2, c[8]));
    v0 = __fadd_rn(v0, o0);
    v1 = __fadd_rn(v1, o1);
    v2 = __fadd_rn(v2, o2);
  }
  g.v[0] = v0;
  g.v[1] = v1;
  g.v[2] = v2;
  float sq = __fadd_rn(__fadd_rn(__fmul_rn(v0, v0), __fmul_rn(v1, v1)), __fmul_rn(v2, v2));
  g.clamped = !(sq > 1e-24f);
  g.r = sqrtf(fmaxf(sq, 1e-24f));
  g.u[0] = v0 / g.r;
  g.u[1] = v1 / g.r;
  g.u[2] = v2 / g.r;
  return g;
}

__device__ __forceinline__ void sh_eval(const float* __restrict__ T, int lmax, const float u[3],
                                        float Y[16]) {
  const float s3 = 1.7320508075688772f;
#pragma unroll
  for (int i = 0; i < 16; ++i) Y[i] = 0.f;
  Y[0] = 1.f;
  if (lmax < 1) return;
  Y[1] = s3 * u[0];
  Y[2] = s3 * u[1];
  Y[3] = s3 * u[2];
  if (lmax < 2) return;
#pragma unroll
  for (int k = 0; k < 5; ++k) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 3; ++i)
#pragma unroll
      for (int j = 0; j < 3; ++j) a += Y[1 + i] * Y[1 + j] * T[(i * 3 + j) * 5 + k];
    Y[4 + k] = a;
  }
  if (lmax < 3) return;
  const float* T3 = T + 45;
#pragma unroll
  for (int k = 0; k < 7; ++k) {
    float a = 0.f;
#pragma unroll
    for (int i = 0; i < 5; ++i)
#pragma unroll
      for (int j = 0; j < 3; ++j) a += Y[4 + i] * Y[1 + j] * T3[(i * 3 + j) * 7 + k];
    Y[9 + k] = a;
  }
}

__device__ __forceinline__ float ipow(float x, int p) {
  float r = 1.f;
  for (int i = 0; i < p; ++i) r *= x;
  return r;
}

constexpr int MAX_NB = 16;

// Bessel argument of edge e: r, or its Agnesi transform (then *drt = dr_t/dr)
__device__ __forceinline__ float bessel_arg(const EdgeParams& p, int64_t e, float r, float* drt) {
  *drt = 1.f;
  if (!p.agnesi) return r;
  const int zs = p.species[p.snd[e]], zr = p.species[p.rcv[e]];
  const float r0 = 0.5f * (__ldg(p.ag_radius + zs) + __ldg(p.ag_radius + zr));
  return agnesi_transform(r, r0, p.ag_q, p.ag_p, p.ag_a, drt);
}

// The recursion tables T2 (45 floats) and T3 (105) in shared memory: every
// thread reads all of them, from the same addresses (broadcast).
constexpr int SH_T_FLOATS = 45 + 105;
__device__ __forceinline__ void stage_sh_tables(const EdgeParams& p, float* sT) {
  const int n = p.max_ell >= 3 ? SH_T_FLOATS : (p.max_ell == 2 ? 45 : 0);
  for (int i = threadIdx.x; i < n; i += blockDim.x) sT[i] = __ldg(p.sh_T + i);
  __syncthreads();
}

__global__ void k_edge_fwd(EdgeParams p) {
  __shared__ float sT[SH_T_FLOATS];
  stage_sh_tables(p, sT);
  int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (e >= p.E) return;
  EdgeGeom g = edge_geom(p, e);
  p.v[3 * e + 0] = g.v[0];
  p.v[3 * e + 1] = g.v[1];
  p.v[3 * e + 2] = g.v[2];
  float Y[16];
  sh_eval(sT, p.max_ell, g.u, Y);
#pragma unroll
  for (int i = 0; i < 16; ++i) p.Y[16 * e + i] = Y[i];
  const float pref = sqrtf(2.0f / p.r_max);
  const float x = g.r / p.r_max;
  const float pf = (float)p.poly_p;
  const float up = ipow(x, p.poly_p);
  float env = 1.0f - ((pf + 1.0f) * (pf + 2.0f) / 2.0f) * up + pf * (pf + 2.0f) * (up * x) -
              (pf * (pf + 1.0f) / 2.0f) * (up * x * x);
  env = (x < 1.0f) ? env : 0.0f;
  float drt;
  const float rb = bessel_arg(p, e, g.r, &drt);
  // envelope on the features, or (envelope_on_weights) kept for the radial-MLP output
  const float bscale = p.cut ? 1.0f : env;
  if (p.cut) p.cut[e] = env;
  for (int n = 0; n < p.nb; ++n) {
    float w = __ldg(p.bessel_w + n);
    float bes = pref * sinf(w * rb) / rb;
    p.b[(int64_t)p.nb * e + n] = bes * bscale;
  }
}

__global__ void k_edge_bwd(EdgeParams p) {
  __shared__ float sT[SH_T_FLOATS];
  stage_sh_tables(p, sT);
  int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  double vir[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) vir[i] = 0.0;
  if (e < p.E) {
    EdgeGeom g = edge_geom(p, e);
    float Y[16];
    sh_eval(sT, p.max_ell, g.u, Y);
    float dYv[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) dYv[i] = p.dY[16 * e + i];
    // back through the recursion Y_l = T_l . (Y_{l-1} x Y_1)
    float dY1[3] = {dYv[1], dYv[2], dYv[3]};
    float dY2[5] = {dYv[4], dYv[5], dYv[6], dYv[7], dYv[8]};
    if (p.max_ell >= 3) {
      const float* T3 = sT + 45;
#pragma unroll
      for (int i = 0; i < 5; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 7; ++k) acc += T3[(i * 3 + j) * 7 + k] * dYv[9 + k];
          dY2[i] += acc * Y[1 + j];
          dY1[j] += acc * Y[4 + i];
        }
    }
    if (p.max_ell >= 2) {
#pragma unroll
      for (int i = 0; i < 3; ++i)
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          float acc = 0.f;
#pragma unroll
          for (int k = 0; k < 5; ++k) acc += sT[(i * 3 + j) * 5 + k] * dY2[k];
          dY1[i] += acc * Y[1 + j];
          dY1[j] += acc * Y[1 + i];
        }
    }
    const float s3 = 1.7320508075688772f;
    float du[3] = {s3 * dY1[0], s3 * dY1[1], s3 * dY1[2]};
    if (p.max_ell < 1) du[0] = du[1] = du[2] = 0.f;
    // radial part
    const float pref = sqrtf(2.0f / p.r_max);
    const float x = g.r / p.r_max;
    const float pf = (float)p.poly_p;
    const float up = ipow(x, p.poly_p);
    const float upm1 = p.poly_p > 0 ? ipow(x, p.poly_p - 1) : 0.f;
    float env = 1.0f - ((pf + 1.0f) * (pf + 2.0f) / 2.0f) * up + pf * (pf + 2.0f) * (up * x) -
                (pf * (pf + 1.0f) / 2.0f) * (up * x * x);
    float denv = -((pf + 1.0f) * (pf + 2.0f) / 2.0f) * pf * upm1 + pf * (pf + 2.0f) * (pf + 1.0f) * up -
                 (pf * (pf + 1.0f) / 2.0f) * (pf + 2.0f) * (up * x);
    denv /= p.r_max;
    if (!(x < 1.0f)) {
      env = 0.f;
      denv = 0.f;
    }
    float drt;
    const float rb = bessel_arg(p, e, g.r, &drt);
    float bes[MAX_NB], dbes[MAX_NB], dbn[MAX_NB];
    for (int n = 0; n < p.nb; ++n) {
      float w = __ldg(p.bessel_w + n);
      float sn, cs;
      sincosf(w * rb, &sn, &cs);
      bes[n] = pref * sn / rb;
      dbes[n] = pref * (w * cs * rb - sn) / (rb * rb) * drt;  // d bes / dr through r_t
      dbn[n] = p.db[(int64_t)p.nb * e + n];
    }
    // density normalisation: d_e = tanh(x^2), x = w_d . b_e, with dE/dD of the receiver
    for (int t = 0; t < p.n_dens; ++t) {
      const float* wd = p.dens_w[t];
      float xd = 0.f;
      for (int n = 0; n < p.nb; ++n) xd = fmaf(__ldg(wd + n), bes[n] * env, xd);
      const float th = tanhf(xd * xd);
      const float gx = p.dD[t][p.rcv[e]] * (1.0f - th * th) * 2.0f * xd;
      for (int n = 0; n < p.nb; ++n) dbn[n] = fmaf(gx, __ldg(wd + n), dbn[n]);
    }
    float dr = 0.f;
    if (p.dcut) {  // b = bare Bessel features; the envelope scaled the radial-MLP output
      for (int n = 0; n < p.nb; ++n) dr += dbn[n] * dbes[n];
      dr = fmaf(p.dcut[e], denv, dr);
    } else {
      for (int n = 0; n < p.nb; ++n) dr += dbn[n] * (dbes[n] * env + bes[n] * denv);
    }
    if (p.zbl) {
      const int s_n = p.snd[e], r_n = p.rcv[e];
      const int zs = p.species[s_n], zr = p.species[r_n];
      float dvdr;
      zbl_pair(g.r, __ldg(p.znum + zs), __ldg(p.znum + zr), __ldg(p.zbl_radius + zs) + __ldg(p.zbl_radius + zr),
               p.zbl_a_exp, p.zbl_a_pref, p.zbl_p, &dvdr);
      const float seed = p.weight ? p.zbl_dscale * p.weight[r_n] : p.zbl_dscale;
      dr = fmaf(seed, dvdr, dr);
    }
    // u = v / r and r = sqrt(max(|v|^2, eps)): dv = (du - u (u.du)) / r + dr * u
    // (when the clamp is active r is a constant and only du / r remains)
    float ud = g.u[0] * du[0] + g.u[1] * du[1] + g.u[2] * du[2];
    float dv[3];
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      float t = du[c] / g.r;
      if (!g.clamped) t += dr * g.u[c] - ud * g.u[c] / g.r;
      dv[c] = t;
    }
    p.dv[3 * e + 0] = dv[0];
    p.dv[3 * e + 1] = dv[1];
    p.dv[3 * e + 2] = dv[2];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
      for (int b = 0; b < 3; ++b) vir[3 * a + b] = (double)g.v[a] * (double)dv[b];
  }
  if (p.virial_part == nullptr) return;
  __shared__ double red[9][256];
#pragma unroll
  for (int i = 0; i < 9; ++i) red[i][threadIdx.x] = vir[i];
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) {
#pragma unroll
      for (int i = 0; i < 9; ++i) red[i][threadIdx.x] += red[i][threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x < 9) p.virial_part[9 * (int64_t)blockIdx.x + threadIdx.x] = red[threadIdx.x][0];
}

// one warp per node: lanes take the node's incoming edges, then a fixed
// shuffle tree sums them (deterministic)
__global__ void k_forces(ForceParams p) {
  const int64_t n = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= p.N) return;
  float f0 = 0.f, f1 = 0.f, f2 = 0.f;
  int bad = 0;
  const int e1 = p.row_ptr[n + 1];
  for (int e = p.row_ptr[n] + lane; e < e1; e += 32) {
    const int r = p.rev[e];
    if (r < 0 || p.snd[r] != (int)n || p.rcv[r] != p.snd[e]) {
      bad = 1;
      continue;
    }
    f0 += p.dv[3 * (int64_t)r + 0] - p.dv[3 * (int64_t)e + 0];
    f1 += p.dv[3 * (int64_t)r + 1] - p.dv[3 * (int64_t)e + 1];
    f2 += p.dv[3 * (int64_t)r + 2] - p.dv[3 * (int64_t)e + 2];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    f0 += __shfl_xor_sync(0xffffffffu, f0, o);
    f1 += __shfl_xor_sync(0xffffffffu, f1, o);
    f2 += __shfl_xor_sync(0xffffffffu, f2, o);
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane != 0) return;
  if (bad) atomicExch(p.err_flag, 1);
  p.forces[3 * n + 0] = f0;
  p.forces[3 * n + 1] = f1;
  p.forces[3 * n + 2] = f2;
}

__global__ void k_virial_reduce(const double* part, int n_part, double* out) {
  __shared__ double red[9][256];
  double acc[9];
#pragma unroll
  for (int i = 0; i < 9; ++i) acc[i] = 0.0;
  for (int b = threadIdx.x; b < n_part; b += blockDim.x)
#pragma unroll
    for (int i = 0; i < 9; ++i) acc[i] += part[9 * (int64_t)b + i];
#pragma unroll
  for (int i = 0; i < 9; ++i) red[i][threadIdx.x] = acc[i];
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w)
#pragma unroll
      for (int i = 0; i < 9; ++i) red[i][threadIdx.x] += red[i][threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x < 9) out[threadIdx.x] = red[threadIdx.x][0];
}

}  // namespace

int launch_edge_fwd(const EdgeParams& p, cudaStream_t s) {
  if (p.E == 0) return MACE_OK;
  if (p.nb > MAX_NB) return fail(MACE_ERR_UNSUPPORTED, "edge features: at most 16 Bessel functions");
  int64_t blocks = (p.E + 255) / 256;
  k_edge_fwd<<<(unsigned)blocks, 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("edge_fwd");
  return MACE_OK;
}

int launch_edge_bwd(const EdgeParams& p, int* n_blocks, cudaStream_t s) {
  int64_t blocks = (p.E + 255) / 256;
  if (blocks == 0) blocks = 1;
  *n_blocks = (int)blocks;
  k_edge_bwd<<<(unsigned)blocks, 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("edge_bwd");
  return MACE_OK;
}

int launch_forces(const ForceParams& p, cudaStream_t s) {
  if (p.N == 0) return MACE_OK;
  k_forces<<<(unsigned)((p.N * 32 + 255) / 256), 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("forces");
  return MACE_OK;
}

int launch_virial_reduce(const double* part, int n_part, double* out, cudaStream_t s) {
  k_virial_reduce<<<1, 256, 0, s>>>(part, n_part, out);
  MACE_LAUNCH_CHECK("virial_reduce");
  return MACE_OK;
}

}  // namespace mace
