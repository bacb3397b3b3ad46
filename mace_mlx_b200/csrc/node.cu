// Node-level ops: o3.Linear (grouped per irrep degree, concat-K), the species-
// indexed skip tensor product, the symmetric contraction and its backward,
// readouts, the one-hot embedding and the energy assembly.
//
// Reference semantics:
//   o3.Linear                      mace_mlx/linear.py:41-77, 421-446
//   skip_tp (uvw with one-hot)     mace_mlx/tensor_product.py:1046-1305
//   symmetric contraction          mace_mlx/symmetric_contraction.py:95-121, 505-595
//   product block                  mace_mlx/blocks.py:493-537
//   readouts                       mace_mlx/blocks.py:540-608
//   energy assembly                mace_mlx/model.py:403-438, 550-589
// Node-feature rows are channel-last per irrep slot (slot offset + m*C + u),
// so a degree-l slot of N nodes is an (N*(2l+1), C) row-major matrix.
#include "common.cuh"

namespace mace {

namespace {

// ---------------------------------------------------------------------------
// o3.Linear: out[(n,m), c] (+)= alpha * sum_{ks,u} in[n, k_off[ks] + m*C + u] * W[ks*C+u][c]
// 64 x 128 output tile per 256-thread CTA, 8 x 4 outputs per thread (32 x 64,
// 2 x 4 per thread, for small node counts); K in
// chunks of 32 through shared memory, the next chunk's loads in flight in
// registers while the current one is multiplied.  Inner step per thread: two
// broadcast 128-bit loads of A, one 128-bit load of B, 32 FMAs.
// With species-indexed weights (the skip tensor product with a one-hot
// species input) the tile runs one pass per distinct species among its rows,
// each with the other rows' A masked to zero: a single pass when the tile's
// nodes share one element.
// ---------------------------------------------------------------------------
constexpr int LK = 32;  // k chunk

// LR x LC output tile per 256-thread CTA (64 x 128, or 32 x 64 with the columns
// split over blockIdx.z when the rows alone would not fill the GPU)
template <int LR, int LC>
__global__ void __launch_bounds__(256) k_linear(LinParams p) {
  constexpr int CT = LC / 4;     // threads across the columns (4 columns each)
  constexpr int RG = 256 / CT;   // row groups
  constexpr int RPT = LR / RG;   // rows per thread
  constexpr int NA = LR / 32;    // float4 of A per thread per chunk
  constexpr int NBQ = LC / 32;   // float4 of B per thread per chunk
  constexpr int LAP = LR + 4;    // pitch of the transposed A tile (16-byte rows, no bank conflicts on the stores)
  static_assert(RPT == 2 || RPT % 4 == 0, "rows per thread");
  __shared__ __align__(16) float sA[LK][LAP];
  __shared__ __align__(16) float sB[LK][LC];
  __shared__ int sZ[LR + 1];  // distinct species of the tile's rows, count in sZ[LR]
  const LinJob& jb = p.job[blockIdx.y];
  const int C = p.C;
  const int rows = (int)(p.N * jb.d);
  const int r0 = blockIdx.x * LR;
  const int col0 = blockIdx.z * LC;
  if (r0 >= rows || col0 >= C) return;
  const int tid = threadIdx.x;
  const int ty = tid / CT, tx = tid % CT;
  // this thread's A row for the loads (fixed across K)
  const int lr = tid % LR, lq = tid / LR;  // row, first 4-wide k group (then + 256 / LR)
  const int arow = r0 + lr;
  const bool arow_in = arow < rows;
  const float* abase = p.in;
  int arow_z = -1;
  if (arow_in) {
    const int node = arow / jb.d, m = arow - node * jb.d;
    abase = p.in + (int64_t)node * p.in_row + m * C;
    if (jb.species) arow_z = jb.species[node];
  }
  int n_pass = 1;
  if (jb.species) {
    if (tid < LR) sZ[tid] = arow_z;
    __syncthreads();
    if (tid == 0) {  // compact the distinct species in place (at most LR)
      int nd = 0;
      for (int q = 0; q < LR; ++q) {
        const int z = sZ[q];
        bool seen = z < 0;
        for (int k = 0; k < nd && !seen; ++k) seen = sZ[k] == z;
        if (!seen) sZ[nd++] = z;
      }
      sZ[LR] = nd;
    }
    __syncthreads();
    n_pass = sZ[LR];
  }
  const int nck = C / LK;
  const int nchunks = jb.n_k * nck;
  bool arow_ok = arow_in;
  const float* wbase = jb.w;
  auto load = [&](int t, float4* ra, float4* rb) {
    const int ks = t / nck, kc = (t - ks * nck) * LK;
    const float* ap = abase + jb.k_off[ks] + kc;
#pragma unroll
    for (int h = 0; h < NA; ++h)
      ra[h] = arow_ok ? __ldg(reinterpret_cast<const float4*>(ap + 4 * (lq + (256 / LR) * h)))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int q = 0; q < NBQ; ++q) {
      const int idx = tid + 256 * q;
      const int kk = idx / CT, c4 = col0 + (idx % CT) * 4;
      rb[q] = (c4 < C) ? __ldg(reinterpret_cast<const float4*>(wbase + (int64_t)(ks * C + kc + kk) * jb.ldb + c4))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  };
  float acc[RPT][4];
#pragma unroll
  for (int a = 0; a < RPT; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  float4 ra[NA], rb[NBQ];
  for (int pass = 0; pass < n_pass; ++pass) {
    if (jb.species) {
      const int z = sZ[pass];
      arow_ok = arow_in && arow_z == z;
      wbase = jb.w + (int64_t)z * jb.zstride;
    }
    load(0, ra, rb);
    for (int t = 0; t < nchunks; ++t) {
#pragma unroll
      for (int h = 0; h < NA; ++h) {
        const int k0 = 4 * (lq + (256 / LR) * h);
        sA[k0 + 0][lr] = ra[h].x;
        sA[k0 + 1][lr] = ra[h].y;
        sA[k0 + 2][lr] = ra[h].z;
        sA[k0 + 3][lr] = ra[h].w;
      }
#pragma unroll
      for (int q = 0; q < NBQ; ++q) {
        const int idx = tid + 256 * q;
        *reinterpret_cast<float4*>(&sB[idx / CT][(idx % CT) * 4]) = rb[q];
      }
      __syncthreads();
      if (t + 1 < nchunks) load(t + 1, ra, rb);
#pragma unroll 8
      for (int kk = 0; kk < LK; ++kk) {
        const float4 b4 = *reinterpret_cast<const float4*>(&sB[kk][tx * 4]);
        float av[RPT];
        if constexpr (RPT == 2) {
          const float2 a2 = *reinterpret_cast<const float2*>(&sA[kk][ty * RPT]);
          av[0] = a2.x;
          av[1] = a2.y;
        } else {
#pragma unroll
          for (int v = 0; v < RPT / 4; ++v) {
            const float4 a4 = *reinterpret_cast<const float4*>(&sA[kk][ty * RPT + 4 * v]);
            av[4 * v + 0] = a4.x;
            av[4 * v + 1] = a4.y;
            av[4 * v + 2] = a4.z;
            av[4 * v + 3] = a4.w;
          }
        }
#pragma unroll
        for (int a = 0; a < RPT; ++a) {
          acc[a][0] = fmaf(av[a], b4.x, acc[a][0]);
          acc[a][1] = fmaf(av[a], b4.y, acc[a][1]);
          acc[a][2] = fmaf(av[a], b4.z, acc[a][2]);
          acc[a][3] = fmaf(av[a], b4.w, acc[a][3]);
        }
      }
      __syncthreads();
    }
  }  // species passes
  const int c = col0 + tx * 4;
  if (c >= C) return;
#pragma unroll
  for (int a = 0; a < RPT; ++a) {
    const int row = r0 + ty * RPT + a;
    if (row >= rows) continue;
    const int node = row / jb.d, m = row - node * jb.d;
    float* const outp = jb.out ? jb.out : p.out;
    const int orow = jb.out ? jb.out_row : p.out_row;
    float4* o = reinterpret_cast<float4*>(outp + (int64_t)node * orow + jb.out_off + m * C + c);
    float4 v = make_float4(jb.alpha * acc[a][0], jb.alpha * acc[a][1], jb.alpha * acc[a][2], jb.alpha * acc[a][3]);
    if (jb.accumulate) {
      const float4 w = *o;
      v.x += w.x;
      v.y += w.y;
      v.z += w.z;
      v.w += w.w;
    }
    *o = v;
  }
}

// ---------------------------------------------------------------------------
// symmetric contraction as a polynomial in the coupling features:
//   out[n][o][M][c] = sum_{entries e of M} G[z_n][e][c] * f[a_e] (* f[b_e] (* f[c_e]))
// (index-symmetrised U pre-contracted with the species weights at load time),
// and its gradient as one polynomial per coupling index k:
//   df[k][c] = sum_e G'[z_n][e][c] * g[r_e][c] (* f[b_e] (* f[c_e])).
// Generic form for any coupling table: one CTA per node, one thread per
// channel, f and g in the thread's own shared-memory column, entries decoded
// at run time, eight independent G loads in flight.  The standard tables
// (16 coupling features, correlation 3) use the generated kernels of
// sc_gen.cu instead.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int ix(int v, int sh) { return (v >> sh) & 15; }

constexpr int SC_UNROLL = 8;

// sum over entries [b, e) of G[q] * f[a] (* f[b] (* f[c])), packed M | a<<4 | b<<8 | c<<12 | nu<<16
__device__ __forceinline__ float sc_poly(const int32_t* __restrict__ ent, const float* __restrict__ G, int C,
                                         const float* f, int b, int e) {
  float acc[SC_UNROLL];
#pragma unroll
  for (int k = 0; k < SC_UNROLL; ++k) acc[k] = 0.f;
  int q = b;
  for (; q + SC_UNROLL <= e; q += SC_UNROLL) {
    int id[SC_UNROLL];
    float g[SC_UNROLL];
#pragma unroll
    for (int k = 0; k < SC_UNROLL; ++k) {
      id[k] = __ldg(ent + q + k);
      g[k] = __ldg(G + (int64_t)(q + k) * C);
    }
#pragma unroll
    for (int k = 0; k < SC_UNROLL; ++k) {
      const int nu = (id[k] >> 16) & 3;
      float v = g[k] * f[ix(id[k], 4) * C];
      if (nu >= 2) v *= f[ix(id[k], 8) * C];
      if (nu >= 3) v *= f[ix(id[k], 12) * C];
      acc[k] += v;
    }
  }
  for (; q < e; ++q) {
    const int id = __ldg(ent + q);
    const int nu = (id >> 16) & 3;
    float v = __ldg(G + (int64_t)q * C) * f[ix(id, 4) * C];
    if (nu >= 2) v *= f[ix(id, 8) * C];
    if (nu >= 3) v *= f[ix(id, 12) * C];
    acc[0] += v;
  }
  float t = 0.f;
#pragma unroll
  for (int k = 0; k < SC_UNROLL; ++k) t += acc[k];
  return t;
}

__global__ void __launch_bounds__(128) k_sc_fwd(ScParams p) {
  extern __shared__ float sf[];  // ncoup x C
  const int C = p.C, c = threadIdx.x;
  const int64_t n = blockIdx.x;
  const int z = p.species[n];
  const int nc = p.ncoup;
  for (int i = 0; i < nc; ++i) sf[i * C + c] = p.f[n * nc * C + i * C + c];
  const float* f = sf + c;
  for (int o = 0; o < p.n_out; ++o) {
    const int L = p.L[o];
    const float* __restrict__ G = p.G[o] + (int64_t)z * p.n_ent[o] * C + c;
    for (int M = 0; M < 2 * L + 1; ++M) {
      const int b = __ldg(p.seg[o] + M), e = __ldg(p.seg[o] + M + 1);
      p.out[n * p.out_row + p.out_off[o] + M * C + c] = sc_poly(p.ent[o], G, C, f, b, e);
    }
  }
}

__global__ void __launch_bounds__(128) k_sc_bwd(ScParams p) {
  extern __shared__ float sm[];
  const int C = p.C, c = threadIdx.x;
  const int64_t n = blockIdx.x;
  const int z = p.species[n];
  const int nc = p.ncoup;
  float* sf = sm;             // ncoup x C (16 rows reserved)
  float* sg = sm + 16 * C;    // product-output gradient rows x C
  for (int i = 0; i < nc; ++i) sf[i * C + c] = p.f[n * nc * C + i * C + c];
  for (int r = 0; r < p.n_rows; ++r) sg[r * C + c] = p.dout[n * p.out_row + r * C + c];
  const float* f = sf + c;
  const float* g = sg + c;
  const float* __restrict__ G = p.Gb + (int64_t)z * p.n_bwd * C + c;
  const int32_t* __restrict__ ent = p.bwd_ent;
  for (int k = 0; k < nc; ++k) {
    const int b = __ldg(p.bwd_seg + k), e = __ldg(p.bwd_seg + k + 1);
    float acc[SC_UNROLL];
#pragma unroll
    for (int u = 0; u < SC_UNROLL; ++u) acc[u] = 0.f;
    int q = b;
    for (; q + SC_UNROLL <= e; q += SC_UNROLL) {
      int id[SC_UNROLL];
      float gw[SC_UNROLL];
#pragma unroll
      for (int u = 0; u < SC_UNROLL; ++u) {
        id[u] = __ldg(ent + q + u);
        gw[u] = __ldg(G + (int64_t)(q + u) * C);
      }
#pragma unroll
      for (int u = 0; u < SC_UNROLL; ++u) {
        const int nu1 = (id[u] >> 8) & 3;
        float v = gw[u] * g[(id[u] >> 10) * C];
        if (nu1 >= 1) v *= f[ix(id[u], 0) * C];
        if (nu1 >= 2) v *= f[ix(id[u], 4) * C];
        acc[u] += v;
      }
    }
    for (; q < e; ++q) {
      const int id = __ldg(ent + q);
      const int nu1 = (id >> 8) & 3;
      float v = __ldg(G + (int64_t)q * C) * g[(id >> 10) * C];
      if (nu1 >= 1) v *= f[ix(id, 0) * C];
      if (nu1 >= 2) v *= f[ix(id, 4) * C];
      acc[0] += v;
    }
    float t = 0.f;
#pragma unroll
    for (int u = 0; u < SC_UNROLL; ++u) t += acc[u];
    p.df[n * nc * C + k * C + c] = t;
  }
}

// ---------------------------------------------------------------------------
// readout of one layer (warp per node) and its gradient seed
// ---------------------------------------------------------------------------
__global__ void k_readout(ReadoutParams p) {
  const int64_t n = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (n >= p.N) return;
  const float* h = p.h + n * p.h_row;
  float* dh = p.dh + n * p.h_row;
  const float dscale = p.weight ? p.dscale * p.weight[n] : p.dscale;
  for (int q = p.C + lane; q < p.h_row; q += 32) dh[q] = 0.f;
  if (!p.nonlinear) {
    float a = 0.f;
    for (int c = lane; c < p.C; c += 32) {
      a = fmaf(h[c], __ldg(p.w1 + c), a);
      dh[c] = dscale * __ldg(p.w1 + c);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) p.e[n] = a;
    return;
  }
  const int H = p.hidden;  // <= 32
  float z = 0.f;
  // z_j for j = lane (lanes >= H idle): the node's scalar row is read once,
  // coalesced, and broadcast by shuffles; the weight loads of 32 channels are
  // independent of one another (C is a multiple of 32, at most 128)
  float hr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) hr[k] = (32 * k < p.C) ? h[32 * k + lane] : 0.f;
  if (H <= 16) {
    // the two half-warps take alternate 16-channel halves of each 32-channel
    // block and add their partial sums: half the dependent chain
    const int j = lane & 15, half = lane >> 4;
    const float* w1j = p.w1 + (j < H ? j : 0);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (32 * k >= p.C) break;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float hv = __shfl_sync(0xffffffffu, hr[k], 16 * half + i);
        z = fmaf(hv, __ldg(w1j + (32 * k + 16 * half + i) * H), z);
      }
    }
    z += __shfl_xor_sync(0xffffffffu, z, 16);
  } else {
    const float* w1l = p.w1 + (lane < H ? lane : 0);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (32 * k >= p.C) break;
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float hv = __shfl_sync(0xffffffffu, hr[k], i);
        z = fmaf(hv, __ldg(w1l + (32 * k + i) * H), z);
      }
    }
  }
  if (lane >= H) z = 0.f;
  float e = 0.f, dz = 0.f;
  if (lane < H) {
    float w2 = __ldg(p.w2 + lane);
    e = silu_f(z) * w2;
    dz = dscale * w2 * silu_grad_f(z);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
  if (lane == 0) p.e[n] = e;
  for (int c = lane; c < p.C; c += 32) {
    float a = 0.f;
    for (int j = 0; j < H; ++j) a = fmaf(__ldg(p.w1 + c * H + j), __shfl_sync(0xffffffffu, dz, j), a);
    dh[c] = a;
  }
}

__global__ void k_embed(EmbedParams p) {
  const int64_t n = blockIdx.x;
  const int z = p.species[n];
  for (int c = threadIdx.x; c < p.C; c += blockDim.x) p.h[n * p.C + c] = __ldg(p.emb + (int64_t)z * p.C + c);
}

__global__ void k_energy(EnergyParams p) {
  __shared__ double red[256];
  const int g = blockIdx.x;
  const int64_t b = p.graph_ptr[g], e = p.graph_ptr[g + 1];
  double acc = 0.0;
  for (int64_t n = b + threadIdx.x; n < e; n += blockDim.x) {
    float inter = 0.f;
    for (int t = 0; t < p.T; ++t) inter += p.e_layers[t * p.N + n];
    float e0 = __ldg(p.e0 + p.species[n]);
    float ne = p.scale_shift ? e0 + (p.scale * inter + p.shift) : e0 + inter;
    if (p.node_energy) p.node_energy[n] = ne;
    acc += p.weight ? (double)p.weight[n] * (double)ne : (double)ne;
  }
  red[threadIdx.x] = acc;
  __syncthreads();
  for (int w = blockDim.x / 2; w > 0; w >>= 1) {
    if ((int)threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
    __syncthreads();
  }
  if (threadIdx.x == 0 && p.energy) p.energy[g] = red[0];
}

}  // namespace

int launch_linear(const LinParams& p, cudaStream_t s) {
  if (p.N == 0 || p.n_jobs == 0) return MACE_OK;
  if (p.C > 128 || p.C % 32 != 0) return fail(MACE_ERR_UNSUPPORTED, "linear: C must be a multiple of 32, <= 128");
  if (p.N * 7 >= (int64_t)1 << 31) return fail(MACE_ERR_UNSUPPORTED, "linear: too many rows");
  if (linear_tc_supported(p)) return launch_linear_tc(p, s);
  int dmax = 1;
  int64_t rows_all = 0;
  for (int j = 0; j < p.n_jobs; ++j) {
    dmax = p.job[j].d > dmax ? p.job[j].d : dmax;
    rows_all += p.N * p.job[j].d;
  }
  if ((rows_all + 63) / 64 >= 148) {  // at least a wave of 64 x 128 tiles
    dim3 grid((unsigned)((p.N * dmax + 63) / 64), (unsigned)p.n_jobs, 1);
    k_linear<64, 128><<<grid, 256, 0, s>>>(p);
  } else {  // small node counts: 32 x 64 tiles, columns split over grid.z
    dim3 grid((unsigned)((p.N * dmax + 31) / 32), (unsigned)p.n_jobs, (unsigned)((p.C + 63) / 64));
    k_linear<32, 64><<<grid, 256, 0, s>>>(p);
  }
  MACE_LAUNCH_CHECK("linear");
  return MACE_OK;
}

// skip_tp with a one-hot species input = per-species (C, C) weights: run as
// species-indexed linear jobs
int skip_jobs(const SkipParams& p, LinJob* jobs) {
  for (int q = 0; q < p.n_jobs; ++q) {
    LinJob& j = jobs[q];
    j = LinJob{};
    j.d = p.d[q];
    j.n_k = 1;
    j.k_off[0] = p.in_off[q];
    j.out_off = p.out_off[q];
    j.ldb = p.C;
    j.w = p.w[q];
    j.alpha = 1.f;
    j.accumulate = p.accumulate;
    j.species = p.species;
    j.zstride = (int64_t)p.C * p.C;
    j.out = p.out;
    j.out_row = p.out_row;
    j.tc = p.tc[q];
  }
  return p.n_jobs;
}

int launch_skip(const SkipParams& p, cudaStream_t s) {
  if (p.N == 0 || p.n_jobs == 0) return MACE_OK;
  LinParams lp{};
  lp.N = p.N;
  lp.C = p.C;
  lp.in = p.in;
  lp.in_row = p.in_row;
  lp.out = p.out;
  lp.out_row = p.out_row;
  lp.n_jobs = skip_jobs(p, lp.job);
  lp.err_flag = p.err_flag;
  return launch_linear(lp, s);
}

int launch_sc_fwd(const ScParams& p, cudaStream_t s) {
  if (p.N == 0) return MACE_OK;
  if (p.gen_sig > 0) {
    bool used = false;
    const int rc = launch_sc_gen(p, p.gen_sig, false, s, &used);
    if (rc || used) return rc;
  }
  if (p.C > 128) return fail(MACE_ERR_UNSUPPORTED, "symmetric contraction: C must be <= 128");
  size_t smem = (size_t)16 * p.C * sizeof(float);
  k_sc_fwd<<<(unsigned)p.N, p.C, smem, s>>>(p);
  MACE_LAUNCH_CHECK("sc_fwd");
  return MACE_OK;
}

int launch_sc_bwd(const ScParams& p, cudaStream_t s) {
  if (p.N == 0) return MACE_OK;
  if (p.gen_sig > 0) {
    bool used = false;
    const int rc = launch_sc_gen(p, p.gen_sig, true, s, &used);
    if (rc || used) return rc;
  }
  if (p.C > 128) return fail(MACE_ERR_UNSUPPORTED, "symmetric contraction: C must be <= 128");
  if (p.n_rows > 48) return fail(MACE_ERR_UNSUPPORTED, "symmetric contraction: product output too wide");
  size_t smem = (size_t)(16 + p.n_rows) * p.C * sizeof(float);
  k_sc_bwd<<<(unsigned)p.N, p.C, smem, s>>>(p);
  MACE_LAUNCH_CHECK("sc_bwd");
  return MACE_OK;
}

int launch_readout(const ReadoutParams& p, cudaStream_t s) {
  if (p.N == 0) return MACE_OK;
  if (p.nonlinear && p.hidden > 32) return fail(MACE_ERR_UNSUPPORTED, "readout hidden width must be <= 32");
  // the non-linear readout holds a node's scalar row in four registers a lane
  if (p.nonlinear && p.C > 128) return fail(MACE_ERR_UNSUPPORTED, "non-linear readout: C must be <= 128");
  int64_t threads = p.N * 32;
  k_readout<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("readout");
  return MACE_OK;
}

int launch_embed(const EmbedParams& p, cudaStream_t s) {
  if (p.N == 0) return MACE_OK;
  k_embed<<<(unsigned)p.N, 128, 0, s>>>(p);
  MACE_LAUNCH_CHECK("embed");
  return MACE_OK;
}

int launch_energy(const EnergyParams& p, cudaStream_t s) {
  if (p.num_graphs == 0) return MACE_OK;
  k_energy<<<(unsigned)p.num_graphs, 256, 0, s>>>(p);
  MACE_LAUNCH_CHECK("energy");
  return MACE_OK;
}

}  // namespace mace
