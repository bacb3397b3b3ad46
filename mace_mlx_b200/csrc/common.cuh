// Internal declarations shared by the CUDA translation units of libmace_b200.
// Not part of the public ABI (include/mace_b200.h is).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/mace_b200.h"

namespace mace {

// ---------------------------------------------------------------------------
// error plumbing (thread-local message, status codes of the C ABI)
// ---------------------------------------------------------------------------
void set_error(const std::string& msg);
int fail(int code, const std::string& msg);

#define MACE_CUDA_TRY(expr)                                                      \
  do {                                                                           \
    cudaError_t _e = (expr);                                                     \
    if (_e != cudaSuccess)                                                       \
      return ::mace::fail(MACE_ERR_CUDA, std::string(#expr) + ": " +            \
                                             cudaGetErrorString(_e));          \
  } while (0)

#define MACE_LAUNCH_CHECK(name)                                                  \
  do {                                                                           \
    cudaError_t _e = cudaGetLastError();                                         \
    if (_e != cudaSuccess)                                                       \
      return ::mace::fail(MACE_ERR_CUDA, std::string("launch ") + name + ": " + \
                                             cudaGetErrorString(_e));          \
  } while (0)

__host__ __device__ __forceinline__ int64_t imin64(int64_t a, int64_t b) { return a < b ? a : b; }

// SiLU with the hardware exponential and reciprocal (__expf, __fdividef):
// a few ulp, about 1e-6 relative at worst for the MLP's pre-activations.
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float silu_grad_f(float x) {
  const float s = __fdividef(1.0f, 1.0f + __expf(-x));
  return s * (1.0f + x * (1.0f - s));
}

// ---------------------------------------------------------------------------
// edge front end
// ---------------------------------------------------------------------------
struct EdgeParams {
  int64_t E;
  const float* pos;
  const float* cell;  // may be null
  const int32_t* snd;
  const int32_t* rcv;
  const int32_t* shifts;
  int max_ell;
  int nb;
  float r_max;
  int poly_p;
  const float* bessel_w;  // (nb)
  const float* sh_T;      // T2 (3*3*5) then T3 (5*3*7)
  float* v;               // (E,3)
  float* Y;               // (E,16)
  float* b;               // (E,nb)
  // envelope_on_weights models: b holds the bare Bessel features, the envelope
  // goes to cut (forward) and dcut is dE/d(envelope) (backward); else both null
  float* cut;             // (E)
  const float* dcut;      // (E)
  // backward
  const float* dY;  // (E,16)
  const float* db;  // (E,nb)
  float* dv;        // (E,3)
  double* virial_part;  // (gridDim, 9)
  // element-dependent terms (mpa-0 family); species gives the element index per node
  const int32_t* species;
  int agnesi;                 // Agnesi transform of the Bessel argument
  float ag_q, ag_p, ag_a;
  const float* ag_radius;     // (num_elements)
  int zbl;                    // ZBL pair repulsion (backward: its gradient)
  int zbl_p;
  float zbl_a_exp, zbl_a_pref;
  const float* zbl_radius;    // (num_elements)
  const float* znum;          // (num_elements) atomic numbers
  float zbl_dscale;           // d(node energy) / d(pair energy): ScaleShiftMACE scale, else 1
  const float* weight;        // (N) energy weight per node, or null (1)
  // density normalisation gradients, one entry per density layer
  int n_dens;
  const float* dens_w[MACE_MAX_LAYERS];  // (nb) density_fn weights
  const float* dD[MACE_MAX_LAYERS];      // (N) dE / d density of the receiver
};
int launch_edge_fwd(const EdgeParams& p, cudaStream_t s);
int launch_edge_bwd(const EdgeParams& p, int* n_blocks, cudaStream_t s);

// Agnesi transform r_t(r) and dr_t/dr (reference radial.py:235-262)
__device__ __forceinline__ float agnesi_transform(float r, float r0, float q, float pp, float a, float* drt_dr) {
  float x = r / r0;
  const bool clamped = !(x > 1e-12f);
  x = clamped ? 1e-12f : x;
  const float xq = powf(x, q), xqp = powf(x, q - pp);
  const float den = 1.0f + xqp;
  const float rt = 1.0f / (1.0f + a * xq / den);
  const float dg_dx = a * (xq / x) * (q + pp * xqp) / (den * den);
  *drt_dr = clamped ? 0.0f : -rt * rt * dg_dx / r0;
  return rt;
}

// polynomial envelope of degree p on u and its derivative (reference radial.py:18-34)
__device__ __forceinline__ float poly_envelope(float u, int p, float* denv_du) {
  const float pf = (float)p;
  float up = 1.f;
  for (int i = 0; i < p - 1; ++i) up *= u;
  const float upm1 = p > 0 ? up : 0.f;  // u^(p-1)
  up = p > 0 ? up * u : 1.f;            // u^p
  float env = 1.0f - ((pf + 1.0f) * (pf + 2.0f) / 2.0f) * up + pf * (pf + 2.0f) * (up * u) -
              (pf * (pf + 1.0f) / 2.0f) * (up * u * u);
  float d = -((pf + 1.0f) * (pf + 2.0f) / 2.0f) * pf * upm1 + pf * (pf + 2.0f) * (pf + 1.0f) * up -
            (pf * (pf + 1.0f) / 2.0f) * (pf + 2.0f) * (up * u);
  if (!(u < 1.0f)) {
    env = 0.f;
    d = 0.f;
  }
  *denv_du = d;
  return env;
}

// ZBL pair energy of one directed edge and its derivative in r (reference radial.py:160-197)
__device__ __forceinline__ float zbl_pair(float r, float zu, float zv, float rmax_pair, float a_exp, float a_pref,
                                          int p, float* dv_dr) {
  const float a = a_pref * 0.529f / (powf(zu, a_exp) + powf(zv, a_exp));
  const float s = r / a;
  const float e1 = expf(-3.2f * s), e2 = expf(-0.9423f * s), e3 = expf(-0.4028f * s), e4 = expf(-0.2016f * s);
  const float phi = 0.1818f * e1 + 0.5099f * e2 + 0.2802f * e3 + 0.02817f * e4;
  const float dphi = -(0.1818f * 3.2f * e1 + 0.5099f * 0.9423f * e2 + 0.2802f * 0.4028f * e3 +
                       0.02817f * 0.2016f * e4) / a;
  const float K = 14.3996f * zu * zv;
  float denv;
  const float env = poly_envelope(r / rmax_pair, p, &denv);
  const float v = 0.5f * (K / r) * phi * env;
  *dv_dr = 0.5f * K * ((dphi / r - phi / (r * r)) * env + (phi / r) * denv / rmax_pair);
  return v;
}

// in-library halo exchange (halo.cu)
int halo_features(mace_halo* h, float* rows, int64_t row_len, cudaStream_t s);
int halo_gradients(mace_halo* h, float* rows, int64_t row_len, cudaStream_t s);
int halo_version(const mace_halo* h);
// A context whose captured step graph holds NCCL operations of halo `h`
// registers itself; destroying the halo first releases those graphs (NCCL
// waits, in ncclCommDestroy, until no graph holds operations of the
// communicator).  ctx_drop_graph releases a context's captured step.
void halo_attach_graph(mace_halo* h, mace_ctx* c);
void halo_detach_graph(mace_halo* h, mace_ctx* c);
void ctx_drop_graph(mace_ctx* c);

// per-node sums over each receiver's edges that need no learned features:
// density of every density layer and the ZBL pair energy (forward), and the
// density rescaling of the interaction message and its gradient
struct NodeSumParams {
  int64_t N;
  const int32_t* row_ptr;
  const int32_t* snd;
  const int32_t* species;
  const float* v;   // (E,3) edge vectors
  const float* b;   // (E,nb) radial basis
  int nb;
  int n_dens;
  const float* dens_w[MACE_MAX_LAYERS];
  float* D[MACE_MAX_LAYERS];  // (N) density per layer
  int zbl;
  int zbl_p;
  float zbl_a_exp, zbl_a_pref;
  const float* zbl_radius;
  const float* znum;
  float* pair;  // (N) pair energy per receiver
};
int launch_node_sums(const NodeSumParams& p, cudaStream_t s);
// rows[n][:] /= (D[n] + 1)
int launch_density_scale(float* rows, int64_t row_len, const float* D, int64_t N, cudaStream_t s);
// dD[n] = -sum_f drows[n][f] rows[n][f] / (D[n] + 1); drows[n][:] *= 1 / (D[n] + 1)
// (rows are the rescaled forward rows)
int launch_density_bwd(const float* rows, float* drows, int64_t row_len, const float* D, float* dD, int64_t N,
                       cudaStream_t s);

struct ForceParams {
  int64_t N;
  const int32_t* row_ptr;
  const int32_t* snd;
  const int32_t* rcv;
  const int32_t* rev;
  const float* dv;
  float* forces;
  int* err_flag;
};
int launch_forces(const ForceParams& p, cudaStream_t s);
int launch_virial_reduce(const double* part, int n_part, double* out, cudaStream_t s);

// ---------------------------------------------------------------------------
// radial MLP
// ---------------------------------------------------------------------------
// Radial weights w and their gradient dw are stored in 128-edge tiles: tile
// e >> 7 holds ceil(W / 32) chunks of 128 rows x 32 floats (16 KB each), and
// inside a chunk row e & 127 fills 128 contiguous bytes whose 16-byte groups
// are XOR-swizzled with (e & 7).  That is the tensor cores' 128B-swizzled
// K-major operand layout, so one chunk moves between HBM and shared memory
// in a single 1-D bulk copy, while a warp reading 32 consecutive columns of
// one edge still reads one 128-byte line.  Rows of the last tile beyond E are
// padding.
constexpr int WT_TILE = 128;
constexpr int WT_CHUNK = WT_TILE * 32;  // floats per chunk
__host__ __device__ __forceinline__ int wt_nchunk(int W) { return (W + 31) / 32; }
__host__ __device__ __forceinline__ int64_t wt_floats(int64_t E, int W) {
  return ((E + WT_TILE - 1) / WT_TILE) * (int64_t)wt_nchunk(W) * WT_CHUNK;
}
__host__ __device__ __forceinline__ int64_t wt_index(int64_t e, int c, int nch) {
  return (((e >> 7) * nch + (c >> 5)) << 12) + ((e & 127) << 5) + ((((c >> 2) & 7) ^ (int)(e & 7)) << 2) + (c & 3);
}

struct MlpParams {
  int64_t E;
  int n_layers;          // Linear layers (last has no activation)
  int widths[8];         // in, hidden..., out
  const float* w[7];     // (in, out) row-major
  const float* wt[7];    // (out, in) row-major
  const float* b;        // (E, widths[0])
  float* act;            // (E, sum hidden) pre-activations of hidden layers
  float* out;            // (E, widths[n_layers]) in 128-edge tiles (wt_index)
  // backward
  const float* dout;     // (E, widths[n_layers]) in 128-edge tiles (wt_index)
  float* db;             // (E, widths[0]) accumulated (+=)
  // tensor-core path (hidden width 64): pre-split, pre-swizzled last-layer images
  const float* tc_img;       // forward chunks (null: CUDA-core path)
  const float* tc_img_bwd;   // backward chunks
  const float* tc_trunk;     // hidden 64 x 64 layers 1.., forward operands
  const float* tc_trunk_bwd; // the same, backward operands
  int* err_flag;             // set to 2 when a bounded wait gives up
  // envelope_on_weights models (else null): the forward scales edge e's output
  // row by cut[e]; the backward first adds dE/d(cut[e]) = (dout . out)[e] / cut[e]
  // into dcut[e] and scales dout's row by cut[e] (both relative to this launch's edges)
  const float* cut;
  float* dcut;
};
int launch_mlp_fwd(const MlpParams& p, cudaStream_t s);
int launch_mlp_bwd(const MlpParams& p, cudaStream_t s);
bool mlp_tc_supported(const MlpParams& p);
int launch_mlp_fwd_tc(const MlpParams& p, cudaStream_t s);
int launch_mlp_bwd_tc(const MlpParams& p, cudaStream_t s);

// ---------------------------------------------------------------------------
// conv tensor product + segmented scatter (receiver CSR)
// ---------------------------------------------------------------------------
struct ConvSlotDev {
  int l1, l2, l3, combo;
  int src_off;   // offset of the x1 slot inside an input row
  int src_ch;    // per-channel offset of x1 slot (sum of dims of earlier input slots)
  int off;       // offset of the slot inside a mid row
  int m_off;     // offset inside a per-edge M row
  int h_off;     // offset (per channel) of the slot's (2l1+1)(2l2+1) H block
  const float* cg;  // (2l1+1)(2l2+1)(2l3+1)
};
struct ConvParams {
  int64_t N;
  int C;
  int n_mid;
  int m_tot;
  int h_tot;     // sum over slots of (2l1+1)(2l2+1)
  int wnumel;
  int wnch;      // wt_nchunk(wnumel)
  int64_t n0;    // first receiver of this launch (blockIdx.x = receiver - n0)
  int64_t e0;    // first edge of the chunk: w / dw hold edges e0.. (tile index of e - e0)
  int in_dim;
  int in_ch;       // in_dim / C
  int mid_dim;
  ConvSlotDev slot[MACE_MAX_MID];
  const int32_t* row_ptr;
  const int32_t* snd;
  const float* Y;        // (E,16)
  const float* up;       // (N,in_dim)
  const float* w;        // (E,wnumel) in 128-edge tiles (wt_index)
  float* A;              // (N,mid_dim)
  // backward
  const float* dA;       // (N,mid_dim)
  float* dw;             // (E,wnumel) in 128-edge tiles (wt_index)
  float* dY;             // (E,16) accumulated
  float* dup;            // (N,in_dim)
  int need_dup;          // 0: the input gradient is not needed (first layer)
  const int32_t* rev;    // (E) reverse edge
  float* tq;             // (E, in_dim) per-edge sender-side terms, or null (then gathered from dA)
  int64_t n_active;      // receivers >= n_active were not evaluated: their sender terms are skipped (0: all)
  // A layer's conv in two launches, each beside part of the radial-MLP tiles:
  // part 1 takes the receivers whose edges lie below e_split (split_first = 0,
  // the forward: all of their edges; 1, the backward: their first edge), part 2
  // the other receivers; split_part 0 takes every receiver.
  int split_part;
  int split_first;
  int64_t e_split;
};
__device__ __forceinline__ bool conv_receiver_skipped(const ConvParams& p, int64_t n) {
  if (!p.split_part) return false;
  const bool below = p.split_first ? p.row_ptr[n] < p.e_split : p.row_ptr[n + 1] <= p.e_split;
  return below != (p.split_part == 1);
}
int launch_conv_fwd(const ConvParams& p, cudaStream_t s);
// *need_gather: the kernel wrote per-edge sender-side terms to p.tq and
// launch_dup_gather must sum them into p.dup
int launch_conv_bwd(const ConvParams& p, cudaStream_t s, bool* need_gather);
int launch_dup_gather(const ConvParams& p, cudaStream_t s);
// layer-signature specialisations (conv_sig.cu); *used = false: not instantiated
int launch_conv_fwd_sig(const ConvParams& p, cudaStream_t s, bool* used);
int launch_conv_bwd_sig(const ConvParams& p, cudaStream_t s, bool* used, bool* need_gather);

// ---------------------------------------------------------------------------
// node-level ops
// ---------------------------------------------------------------------------
struct LinJob {
  int d;            // 2l+1 rows per node
  int n_k;          // number of C-wide input slots (concat-K)
  int k_off[MACE_MAX_SRC];
  int out_off;
  int ldb;          // row stride of the weight matrix
  const float* w;   // (n_k*C, ldb) row-major, first C columns used
  float alpha;
  int accumulate;
  // species-indexed weights (skip_tp): row (n, m) uses w + species[n] * zstride
  const int32_t* species;
  int64_t zstride;
  // this job's output rows, or null for LinParams::out / out_row
  float* out;
  int out_row;
  // tensor-core operand image of w (launch_tc_image), or null (CUDA cores)
  const float* tc;
};
struct LinParams {
  int64_t N;
  int C;
  const float* in;
  int in_row;
  float* out;
  int out_row;
  int n_jobs;
  LinJob job[MACE_MAX_MID];
  int* err_flag;  // device error flag (tensor-core wait timeouts), may be null
};
// device error flag values of the tensor-core kernels
constexpr int TC_ERR_TIMEOUT = 2;  // an mbarrier wait gave up
constexpr int TC_ERR_ALIGN = 8;    // dynamic shared memory not 1024-byte aligned
// the tensor-core kernel when every job has an image (linear_tc.cu), else CUDA cores
int launch_linear(const LinParams& p, cudaStream_t s);
bool linear_tc_supported(const LinParams& p);
int launch_linear_tc(const LinParams& p, cudaStream_t s);
// operand image of the first N columns of the (K x ldb) row-major weight w
// (Z species blocks zstride apart): tc_image_floats(K, N, Z) floats at img
int64_t tc_image_floats(int K, int N, int Z);
int launch_tc_image(const float* w, int K, int ldb, int N, int Z, int64_t zstride, float* img, cudaStream_t s);

struct SkipParams {
  int64_t N;
  int C;
  const int32_t* species;
  const float* in;
  int in_row;
  float* out;
  int out_row;
  int n_jobs;
  int d[MACE_MAX_IN];
  int in_off[MACE_MAX_IN];
  int out_off[MACE_MAX_IN];
  const float* w[MACE_MAX_IN];  // (num_elements, C, C)
  const float* tc[MACE_MAX_IN];  // their tensor-core images, or null
  int accumulate;
  int* err_flag;
};
int launch_skip(const SkipParams& p, cudaStream_t s);
// the skip_tp jobs of p as species-indexed linear jobs writing p.out (returns the count)
int skip_jobs(const SkipParams& p, LinJob* jobs);

struct ScParams {
  int64_t N;
  int C;
  const int32_t* species;
  const float* f;   // (N, ncoup*C) coupling-major rows
  int ncoup;        // (max_ell+1)^2
  int n_out;
  int L[MACE_MAX_IN];
  int out_off[MACE_MAX_IN];
  int n_ent[MACE_MAX_IN];
  const int32_t* seg[MACE_MAX_IN];  // (2L+2) entry segment starts by M
  const int32_t* ent[MACE_MAX_IN];  // packed M | a<<4 | b<<8 | c<<12 | nu<<16
  const float* G[MACE_MAX_IN];      // (num_elements, n_ent, C)
  float* out;       // (N, out_row)
  int out_row;
  // backward
  const float* dout;
  float* df;        // (N, ncoup*C)
  int n_bwd;                 // backward polynomial, one segment per coupling index
  const int32_t* bwd_seg;    // (ncoup + 1)
  const int32_t* bwd_ent;    // packed b | c<<4 | nu'<<8 | r<<10
  const float* Gb;           // (num_elements, n_bwd, C)
  int n_rows;                // rows of the product output (hid.dim / C)
  int gen_sig;               // > 0: generated kernels of sc_gen.cu apply (signature id)
};
// generated straight-line kernels (sc_gen.cu); *used = false: not available for p.C
int launch_sc_gen(const ScParams& p, int sig, bool bwd, cudaStream_t s, bool* used);
int launch_sc_fwd(const ScParams& p, cudaStream_t s);
int launch_sc_bwd(const ScParams& p, cudaStream_t s);

struct ReadoutParams {
  int64_t N;
  int C;
  const float* h;
  int h_row;
  int nonlinear;
  int hidden;
  const float* w1;
  const float* w2;
  float* e;       // (N) readout energy of this layer
  float* dh;      // (N, h_row) gradient seed (overwritten; zero outside the 0e slot)
  float dscale;   // dE/d e
  const float* weight;  // (N) energy weight per node, or null (1)
};
int launch_readout(const ReadoutParams& p, cudaStream_t s);

struct EmbedParams {
  int64_t N;
  int C;
  const int32_t* species;
  const float* emb;
  float* h;
};
int launch_embed(const EmbedParams& p, cudaStream_t s);

struct EnergyParams {
  int64_t N;
  int num_graphs;
  int T;
  const int32_t* species;
  const int32_t* graph_ptr;
  const float* e0;
  const float* e_layers;  // (T, N)
  int scale_shift;
  float scale, shift;
  float* node_energy;
  double* energy;
  const float* weight;  // (N) energy weight per node, or null (1)
};
int launch_energy(const EnergyParams& p, cudaStream_t s);

// ---------------------------------------------------------------------------
// neighbour list
// ---------------------------------------------------------------------------
struct NlParams {
  int64_t n;
  const double* pos;
  const double* cell;
  const double* inv_cell;  // device (9)
  int pbc[3];
  double r_cut;
  double reach[3];  // r_cut / (perpendicular width) per axis
  const int32_t* graph_ptr;
  int num_graphs;
  const int32_t* node_graph;  // (n)
  const int32_t* wrap;        // (n,3) floor of fractional coordinates
  int32_t* count;             // (n+1)
  int32_t* row_ptr;
  int32_t* snd;
  int32_t* rcv;
  int32_t* shifts;
  int32_t* rev;
  int* err_flag;
  // cell lists (mode 1) or every pair of a graph (mode 0).  Bin coordinates
  // are fractional when the system has a cell (use_frac), else Cartesian;
  // periodic axes bin the wrapped coordinate in [0, 1) and wrap around, open
  // axes bin [origin, origin + nbin / inv_binw) and end there.
  int mode;
  int use_frac;
  int nbin[3];
  double origin[3], inv_binw[3];
  int32_t* atom_bin;   // (n)
  int32_t* bin_start;  // (nbins + 1)
  int32_t* bin_fill;   // (nbins)
  int32_t* bin_atoms;  // (n) atom ids ordered by bin
  unsigned long long* keys;  // (capacity) unsorted (sender, S) keys of the fill pass
};
constexpr int NL_SHIFT_RANGE = 511;  // cell-list keys hold |S| <= 511 per axis
constexpr int NL_ERR_SHIFT = 2;      // err_flag value: a cell-list shift out of range
int launch_nl_bins(const NlParams& p, void* tmp, size_t tmp_bytes, cudaStream_t s);
int launch_nl_cl_count(const NlParams& p, cudaStream_t s);
int launch_nl_cl_fill(const NlParams& p, cudaStream_t s);
int launch_nl_bbox(const NlParams& p, double* out6, cudaStream_t s);
int launch_nl_prep(const NlParams& p, int32_t* node_graph, int32_t* wrap, cudaStream_t s);
int launch_nl_count(const NlParams& p, cudaStream_t s);
int launch_nl_fill(const NlParams& p, cudaStream_t s);
int launch_nl_rev(const NlParams& p, int64_t E, cudaStream_t s);
int scan_counts(int32_t* count, int32_t* row_ptr, int64_t n, void* tmp, size_t tmp_bytes,
                cudaStream_t s);
size_t scan_tmp_bytes(int64_t n);

}  // namespace mace
