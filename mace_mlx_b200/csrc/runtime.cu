// Context, workspace and the C ABI of libmace_b200 (include/mace_b200.h).
//
// mace_forward_backward issues, on one stream, the whole energy + forces
// (+ virial) step: edge features, then per interaction layer the node linears,
// radial MLP, conv tensor product with receiver-segmented sum, symmetric
// contraction, product linear and readout; then the hand-written backward in
// reverse layer order, the edge backward, and the force/virial assembly.  It
// replaces the reference's mx.value_and_grad step (calculators.py:431-483,
// 533-570) with explicit kernels; nothing is allocated on this path.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace mace {

static thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

}  // namespace mace

using namespace mace;

namespace {

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

struct LayerBufs {
  float* up = nullptr;    // (N, in_dim)
  float* w = nullptr;     // (E, wnumel) in 128-edge tiles
  float* act = nullptr;   // (E, nh*H)
  float* A = nullptr;     // (N, mid_dim)
  float* msg = nullptr;   // (N, 16C)
  float* msg2 = nullptr;  // (N, 16C) non-residual skip output
  float* B = nullptr;     // (N, hid_dim)
  float* dB = nullptr;    // (N, hid_dim)
  float* dmsg = nullptr;  // (N, 16C)
  float* dmsg2 = nullptr; // (N, 16C)
  float* dA = nullptr;    // (N, mid_dim)
  float* dup = nullptr;   // (N, in_dim)
};

}  // namespace

struct mace_ctx {
  int device = 0;
  int sm_count = 0;  // multiprocessors of the device (queried on first use)
  mace_model_desc desc{};
  float* d_floats = nullptr;
  int32_t* d_ints = nullptr;
  int64_t cap_nodes = 0, cap_edges = 0;
  int64_t cap_chunk_edges = 0;  // edges of one receiver chunk the radial-weight buffers hold
  std::vector<void*> allocs;
  int64_t ws_bytes = 0;
  // edge buffers
  float *v = nullptr, *Y = nullptr, *b = nullptr, *dY = nullptr, *db = nullptr, *dv = nullptr,
        *dw = nullptr;
  float *cut = nullptr, *dcut = nullptr;  // (E) envelope and its gradient (envelope_on_weights models)
  double* vir_part = nullptr;
  // node buffers
  std::vector<float*> h;   // h[t], t = 0..T   (N, row_t)
  std::vector<float*> dh;  // dh[t]
  std::vector<int> h_row;
  float* e_layers = nullptr;  // (T, N), then the ZBL pair energies (N) when the model has them
  float* dens = nullptr;      // (T, N) density of every density-normalised layer
  float* ddens = nullptr;     // (T, N) its gradient
  LayerBufs lb[MACE_MAX_LAYERS];
  // neighbour-list scratch
  int32_t *nl_count = nullptr, *nl_graph = nullptr, *nl_wrap = nullptr;
  double* nl_inv = nullptr;
  // cell-list scratch: bins for up to nl_bin_cap bins, unsorted edge keys
  int32_t *nl_atom_bin = nullptr, *nl_bin_start = nullptr, *nl_bin_fill = nullptr, *nl_bin_atoms = nullptr;
  int64_t nl_bin_cap = 0;
  double* nl_bbox = nullptr;
  unsigned long long* nl_keys = nullptr;
  int64_t nl_keys_cap = 0;
  void* scan_tmp = nullptr;
  size_t scan_bytes = 0;
  int* d_err = nullptr;
  // MACE_B200_MLP_CUDA_CORES=1 at context creation selects the CUDA-core MLP kernels
  bool mlp_cuda_cores = false;
  // MACE_B200_SINGLE_STREAM=1 at context creation keeps every kernel on the
  // caller's stream (no radial-MLP fork)
  bool single_stream = false;
  // tensor-core operand images of the node-linear weights, by weight pointer
  // (MACE_B200_LINEAR_CUDA_CORES=1 at context creation leaves them out, which
  // keeps the node linears on the CUDA cores)
  float* tc_images = nullptr;
  std::vector<std::pair<const float*, const float*>> tc_index;
  // bookkeeping
  int launches = 0;
  int64_t last_N = 0, last_E = 0;
  // opt-in per-launch timing with CUDA events on the launching stream
  static constexpr int PROF_MAX = 256;
  bool prof_on = false;
  int prof_n = 0;
  cudaEvent_t ev[2 * PROF_MAX] = {};
  const char* prof_name[PROF_MAX] = {};
  int prof_layer[PROF_MAX] = {};
  int prof_stream[PROF_MAX] = {};
  // the last folded step's launches: start and end relative to its first launch
  struct ProfSpan {
    std::string name;
    int layer;
    int stream;
    float t0, t1;
  };
  std::vector<ProfSpan> prof_last;
  struct ProfAcc {
    std::string name;
    int layer;
    int count;
    double ms;
  };
  std::vector<ProfAcc> prof_acc;
  // CUDA-graph replay of the whole step, keyed on the exact call arguments
  cudaStream_t cap_stream = nullptr;
  // second stream for the radial-MLP chain (forked from and joined into the step's stream)
  cudaStream_t aux = nullptr;
  static constexpr int NEV = 6 * MACE_MAX_LAYERS + 4;  // indices up to 4 + 5 T (forward_backward)
  cudaEvent_t fork_ev[NEV] = {};
  // per-layer dW buffers (when the whole list fits one chunk), so that one
  // layer's MLP backward can overlap the next layer's conv backward
  float* dw_layer[MACE_MAX_LAYERS] = {};
  // per-edge sender-side terms of the conv backward (one chunk only), or null
  float* tq = nullptr;
  cudaGraphExec_t gexec = nullptr;
  mace_system g_sys{};
  mace_outputs g_out{};
  int g_flags = -1;
  std::vector<int64_t> g_chunks;  // chunk boundaries of the captured call (host arrays)
  int g_launches = 0;
  int g_halo_version = 0;  // plan version of the captured step's halo exchange
  mace_halo* g_halo = nullptr;  // the halo whose NCCL operations the captured step holds
  // profiling inside the graph: its event-record nodes fill the first g_prof_n slots
  bool g_prof = false;
  int g_prof_n = 0;
};

namespace {

const float* F(const mace_ctx* c, int64_t off) { return c->d_floats + off; }
const int32_t* I(const mace_ctx* c, int64_t off) { return c->d_ints + off; }

int max_wnumel(const mace_model_desc& d) {
  int m = 0;
  for (int t = 0; t < d.num_layers; ++t) m = d.layers[t].wnumel > m ? d.layers[t].wnumel : m;
  return m;
}

// release the captured step (and its registration with the halo it holds)
void drop_graph(mace_ctx* c) {
  if (c->gexec) cudaGraphExecDestroy(c->gexec);
  c->gexec = nullptr;
  if (c->g_halo) halo_detach_graph(c->g_halo, c);
  c->g_halo = nullptr;
}

void free_ws(mace_ctx* c) {
  drop_graph(c);  // a captured step refers to the workspace being released
  for (void* p : c->allocs) cudaFree(p);
  c->allocs.clear();
  if (c->nl_keys) cudaFree(c->nl_keys);
  c->nl_keys = nullptr;
  c->nl_keys_cap = 0;
  c->ws_bytes = 0;
  c->cap_nodes = c->cap_edges = 0;
}

template <typename T>
int alloc(mace_ctx* c, T** p, int64_t count) {
  size_t bytes = (size_t)(count > 0 ? count : 1) * sizeof(T);
  bytes = (bytes + 255) & ~(size_t)255;
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes);
  if (e != cudaSuccess) return fail(MACE_ERR_CUDA, std::string("workspace cudaMalloc: ") + cudaGetErrorString(e));
  c->allocs.push_back(q);
  c->ws_bytes += (int64_t)bytes;
  *p = reinterpret_cast<T*>(q);
  return MACE_OK;
}

#define TRY(x)              \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

// fold recorded event pairs into the per-(kernel, layer) totals
int prof_fold(mace_ctx* c) {
  if (c->prof_n == 0) return MACE_OK;
  MACE_CUDA_TRY(cudaEventSynchronize(c->ev[2 * c->prof_n - 1]));
  for (int i = 0; i < c->prof_n; ++i) MACE_CUDA_TRY(cudaEventSynchronize(c->ev[2 * i + 1]));
  c->prof_last.clear();
  for (int i = 0; i < c->prof_n; ++i) {
    float ms = 0.f, t0 = 0.f, t1 = 0.f;
    MACE_CUDA_TRY(cudaEventElapsedTime(&ms, c->ev[2 * i], c->ev[2 * i + 1]));
    MACE_CUDA_TRY(cudaEventElapsedTime(&t0, c->ev[0], c->ev[2 * i]));
    MACE_CUDA_TRY(cudaEventElapsedTime(&t1, c->ev[0], c->ev[2 * i + 1]));
    c->prof_last.push_back({c->prof_name[i], c->prof_layer[i], c->prof_stream[i], t0, t1});
    bool found = false;
    for (auto& a : c->prof_acc)
      if (a.layer == c->prof_layer[i] && a.name == c->prof_name[i]) {
        a.count += 1;
        a.ms += ms;
        found = true;
        break;
      }
    if (!found) c->prof_acc.push_back({c->prof_name[i], c->prof_layer[i], 1, (double)ms});
  }
  c->prof_n = 0;
  return MACE_OK;
}

// every kernel launch of the step goes through here: counted, and timed when profiling
template <class Fn>
int launch(mace_ctx* c, const char* name, int layer, cudaStream_t s, Fn&& fn) {
  ++c->launches;
  int slot = -1;
  if (c->prof_on && c->prof_n < mace_ctx::PROF_MAX) {
    slot = c->prof_n++;
    c->prof_name[slot] = name;
    c->prof_layer[slot] = layer;
    c->prof_stream[slot] = (s == c->aux && c->aux) ? 1 : 0;
  }
  // inside a stream capture the records must be external to become
  // event-record nodes of the graph; outside one that flag is refused
  unsigned rec_flags = cudaEventRecordDefault;
  if (slot >= 0) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    MACE_CUDA_TRY(cudaStreamIsCapturing(s, &cs));
    if (cs == cudaStreamCaptureStatusActive) rec_flags = cudaEventRecordExternal;
    MACE_CUDA_TRY(cudaEventRecordWithFlags(c->ev[2 * slot], s, rec_flags));
  }
  int rc = fn();
  if (slot >= 0) MACE_CUDA_TRY(cudaEventRecordWithFlags(c->ev[2 * slot + 1], s, rec_flags));
  return rc;
}

#define LAUNCH(name, layer, expr) TRY(launch(c, name, layer, s, [&]() { return (expr); }))
#define LAUNCH_ON(st, name, layer, expr) TRY(launch(c, name, layer, st, [&]() { return (expr); }))

int reserve(mace_ctx* c, int64_t N, int64_t E, int64_t EC) {
  const mace_model_desc& d = c->desc;
  free_ws(c);
  const int C = d.C;
  const int T = d.num_layers;
  const int wmax = max_wnumel(d);
  TRY(alloc(c, &c->v, E * 3));
  TRY(alloc(c, &c->Y, E * 16));
  TRY(alloc(c, &c->b, E * d.num_bessel));
  TRY(alloc(c, &c->dY, E * 16));
  TRY(alloc(c, &c->db, E * d.num_bessel));
  TRY(alloc(c, &c->dv, E * 3));
  c->cut = c->dcut = nullptr;
  if (d.envelope_on_weights) {
    TRY(alloc(c, &c->cut, E));
    TRY(alloc(c, &c->dcut, E));
  }
  TRY(alloc(c, &c->dw, wt_floats(EC, wmax)));
  // padding rows of the last edge tile are read (never used) by the MLP backward
  if (cudaMemset(c->dw, 0, (size_t)wt_floats(EC, wmax) * sizeof(float)) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess)
    return fail(MACE_ERR_CUDA, "workspace memset");
  for (int t = 0; t < T; ++t) c->dw_layer[t] = nullptr;
  c->tq = nullptr;
  if (EC >= E && T > 1) {
    int in_max = 0;
    for (int t = 1; t < T; ++t) in_max = d.layers[t].in.dim > in_max ? d.layers[t].in.dim : in_max;
    TRY(alloc(c, &c->tq, E * in_max));
    for (int t = 0; t < T; ++t) {
      const int64_t n = wt_floats(EC, d.layers[t].wnumel);
      TRY(alloc(c, &c->dw_layer[t], n));
      if (cudaMemset(c->dw_layer[t], 0, (size_t)n * sizeof(float)) != cudaSuccess)
        return fail(MACE_ERR_CUDA, "workspace memset");
    }
  }
  TRY(alloc(c, &c->vir_part, ((E + 255) / 256 + 1) * 9));
  c->h.assign(T + 1, nullptr);
  c->dh.assign(T + 1, nullptr);
  c->h_row.assign(T + 1, 0);
  c->h_row[0] = C;
  for (int t = 0; t < T; ++t) c->h_row[t + 1] = d.layers[t].hid.dim;
  for (int t = 0; t <= T; ++t) {
    TRY(alloc(c, &c->h[t], N * c->h_row[t]));
    TRY(alloc(c, &c->dh[t], N * c->h_row[t]));
  }
  TRY(alloc(c, &c->e_layers, (int64_t)(T + 1) * N));
  TRY(alloc(c, &c->dens, (int64_t)T * N));
  TRY(alloc(c, &c->ddens, (int64_t)T * N));
  for (int t = 0; t < T; ++t) {
    const mace_layer_desc& L = d.layers[t];
    LayerBufs& B = c->lb[t];
    int nh = L.n_mlp - 1, H = L.mlp_w[1];
    TRY(alloc(c, &B.up, N * L.in.dim));
    TRY(alloc(c, &B.w, wt_floats(EC, L.wnumel)));
    TRY(alloc(c, &B.act, EC * nh * H));
    TRY(alloc(c, &B.A, N * L.mid.dim));
    TRY(alloc(c, &B.msg, N * L.inter.dim));
    TRY(alloc(c, &B.B, N * L.hid.dim));
    TRY(alloc(c, &B.dB, N * L.hid.dim));
    TRY(alloc(c, &B.dmsg, N * L.inter.dim));
    TRY(alloc(c, &B.dA, N * L.mid.dim));
    TRY(alloc(c, &B.dup, N * L.in.dim));
    if (!L.residual) {
      TRY(alloc(c, &B.msg2, N * L.inter.dim));
      TRY(alloc(c, &B.dmsg2, N * L.inter.dim));
    }
  }
  TRY(alloc(c, &c->nl_count, N + 1));
  TRY(alloc(c, &c->nl_graph, N));
  TRY(alloc(c, &c->nl_wrap, N * 3));
  TRY(alloc(c, &c->nl_inv, 9));
  c->nl_bin_cap = 2 * N + 64;
  TRY(alloc(c, &c->nl_atom_bin, N));
  TRY(alloc(c, &c->nl_bin_atoms, N));
  TRY(alloc(c, &c->nl_bin_start, c->nl_bin_cap + 1));
  TRY(alloc(c, &c->nl_bin_fill, c->nl_bin_cap + 1));
  TRY(alloc(c, &c->nl_bbox, 6));
  c->scan_bytes = scan_tmp_bytes(c->nl_bin_cap + 1 > N + 1 ? c->nl_bin_cap : N);
  TRY(alloc(c, reinterpret_cast<char**>(&c->scan_tmp), (int64_t)c->scan_bytes));
  TRY(alloc(c, &c->d_err, 1));
  MACE_CUDA_TRY(cudaMemset(c->d_err, 0, sizeof(int)));
  c->cap_nodes = N;
  c->cap_edges = E;
  c->cap_chunk_edges = EC;
  return MACE_OK;
}

// ---------------------------------------------------------------------------
// job builders for the node linears
// ---------------------------------------------------------------------------
const float* tc_find(const mace_ctx* c, const float* w) {
  for (const auto& e : c->tc_index)
    if (e.first == w) return e.second;
  return nullptr;
}

LinJob make_job(const mace_ctx* c, int d, int n_k, const int* k_off, int out_off, const float* w, int ldb,
                float alpha, int accumulate) {
  LinJob j{};
  j.tc = tc_find(c, w);
  j.d = d;
  j.n_k = n_k;
  for (int q = 0; q < n_k; ++q) j.k_off[q] = k_off[q];
  j.out_off = out_off;
  j.w = w;
  j.ldb = ldb;
  j.alpha = alpha;
  j.accumulate = accumulate;
  return j;
}

int run_linear_slots(mace_ctx* c, const char* name, int layer, int64_t N, const mace_slots& in_slots,
                     const mace_slots& out_slots, const int64_t* f_w, const float* in, float* out,
                     int accumulate, cudaStream_t s) {
  // 1-to-1 linears: slot q of `in_slots` -> slot q of `out_slots`
  LinParams p{};
  p.N = N;
  p.C = c->desc.C;
  p.in = in;
  p.in_row = in_slots.dim;
  p.out = out;
  p.out_row = out_slots.dim;
  p.n_jobs = in_slots.n;
  p.err_flag = c->d_err;
  for (int q = 0; q < in_slots.n; ++q) {
    int ko = in_slots.off[q];
    p.job[q] = make_job(c, 2 * in_slots.l[q] + 1, 1, &ko, out_slots.off[q], F(c, f_w[q]), p.C, 1.f, accumulate);
  }
  return launch(c, name, layer, s, [&]() { return launch_linear(p, s); });
}

ConvParams conv_params(mace_ctx* c, int t, int64_t N, const mace_system* sys) {
  const mace_layer_desc& L = c->desc.layers[t];
  ConvParams p{};
  p.N = N;
  p.C = L.C;
  p.n_mid = L.n_mid;
  p.m_tot = L.m_tot;
  p.wnumel = L.wnumel;
  p.wnch = wt_nchunk(L.wnumel);
  p.in_dim = L.in.dim;
  p.in_ch = L.in.dim / L.C;
  p.mid_dim = L.mid.dim;
  p.h_tot = 0;
  for (int k = 0; k < L.n_mid; ++k) {
    const mace_conv_slot& cs = L.conv[k];
    ConvSlotDev& d = p.slot[k];
    d.h_off = p.h_tot;
    p.h_tot += (2 * cs.l1 + 1) * (2 * cs.l2 + 1);
    d.l1 = cs.l1;
    d.l2 = cs.l2;
    d.l3 = cs.l3;
    d.combo = cs.l1 * 16 + cs.l2 * 4 + cs.l3;
    d.src_off = L.in.off[cs.src];
    d.src_ch = L.in.off[cs.src] / L.C;
    d.off = cs.off;
    d.m_off = cs.m_off;
    d.cg = F(c, cs.f_cg);
  }
  p.row_ptr = sys->row_ptr;
  p.snd = sys->sender;
  p.Y = c->Y;
  p.up = c->lb[t].up;
  p.w = c->lb[t].w;
  p.A = c->lb[t].A;
  p.dA = c->lb[t].dA;
  p.dw = c->dw_layer[t] ? c->dw_layer[t] : c->dw;
  p.dY = c->dY;
  p.dup = c->lb[t].dup;
  p.need_dup = t > 0;
  p.rev = sys->rev;
  p.tq = c->tq;
  return p;
}

// radial MLP over edges e0 .. e0 + ne (the chunk's weights are in the layer buffers)
MlpParams mlp_params(mace_ctx* c, int t, int64_t e0, int64_t ne) {
  const mace_layer_desc& L = c->desc.layers[t];
  MlpParams p{};
  p.E = ne;
  p.n_layers = L.n_mlp;
  for (int j = 0; j <= L.n_mlp; ++j) p.widths[j] = L.mlp_w[j];
  for (int j = 0; j < L.n_mlp; ++j) {
    p.w[j] = F(c, L.f_mlp[j]);
    p.wt[j] = F(c, L.f_mlp_t[j]);
  }
  p.b = c->b + e0 * c->desc.num_bessel;
  p.act = c->lb[t].act;
  p.out = c->lb[t].w;
  p.dout = c->dw_layer[t] ? c->dw_layer[t] : c->dw;
  p.db = c->db + e0 * c->desc.num_bessel;
  if (c->desc.envelope_on_weights) {
    p.cut = c->cut + e0;
    p.dcut = c->dcut + e0;
  }
  const bool tc_ok = !c->mlp_cuda_cores && L.f_mlp_tc >= 0 && L.f_mlp_tc_bwd >= 0 && L.f_mlp_tc_trunk >= 0 &&
                     L.f_mlp_tc_trunk_bwd >= 0;
  p.tc_img = tc_ok ? F(c, L.f_mlp_tc) : nullptr;
  p.tc_img_bwd = tc_ok ? F(c, L.f_mlp_tc_bwd) : nullptr;
  p.tc_trunk = tc_ok ? F(c, L.f_mlp_tc_trunk) : nullptr;
  p.tc_trunk_bwd = tc_ok ? F(c, L.f_mlp_tc_trunk_bwd) : nullptr;
  p.err_flag = c->d_err;
  return p;
}

// MLP launch over edges [e0, e0 + ne) of the whole-list buffers (e0 a multiple
// of the 128-edge tile): its rows of every per-edge array and its tiles of
// the radial weights and their gradient
MlpParams mlp_params_tiles(mace_ctx* c, int t, int64_t e0, int64_t ne) {
  MlpParams p = mlp_params(c, t, e0, ne);
  const mace_layer_desc& L = c->desc.layers[t];
  int64_t act_row = 0;
  for (int j = 1; j < L.n_mlp; ++j) act_row += L.mlp_w[j];
  const int64_t tile_floats = (int64_t)wt_nchunk(L.mlp_w[L.n_mlp]) * WT_CHUNK;
  p.act += e0 * act_row;
  p.out += (e0 / WT_TILE) * tile_floats;
  p.dout += (e0 / WT_TILE) * tile_floats;
  return p;
}

ScParams sc_params(mace_ctx* c, int t, int64_t N, const int32_t* species, const float* f, float* out,
                   const float* dout, float* df) {
  const mace_layer_desc& L = c->desc.layers[t];
  ScParams p{};
  p.N = N;
  p.C = L.C;
  p.species = species;
  p.f = f;
  p.ncoup = L.inter.dim / L.C;
  p.n_out = L.hid.n;
  p.out = out;
  p.out_row = L.hid.dim;
  p.dout = dout;
  p.df = df;
  for (int o = 0; o < L.hid.n; ++o) {
    const mace_sc_out& so = L.sc[o];
    p.L[o] = so.L;
    p.out_off[o] = L.hid.off[o];
    p.n_ent[o] = so.n_ent;
    p.seg[o] = I(c, so.i_ent);
    p.ent[o] = I(c, so.i_ent) + (2 * so.L + 2);
    p.G[o] = F(c, so.f_G);
  }
  p.n_bwd = L.sc_n_bwd;
  p.bwd_seg = I(c, L.i_sc_bwd);
  p.bwd_ent = I(c, L.i_sc_bwd) + p.ncoup + 1;
  p.Gb = F(c, L.f_sc_bwd);
  p.n_rows = L.hid.dim / L.C;
  p.gen_sig = L.sc_gen;
  return p;
}

SkipParams skip_params(mace_ctx* c, int t, int64_t N, const int32_t* species, bool transpose,
                       const mace_slots& in_s, const mace_slots& out_s, const float* in, float* out,
                       int accumulate) {
  const mace_layer_desc& L = c->desc.layers[t];
  SkipParams p{};
  p.N = N;
  p.C = L.C;
  p.species = species;
  p.n_jobs = L.n_skip;
  p.in = in;
  p.out = out;
  p.accumulate = accumulate;
  p.err_flag = c->d_err;
  p.in_row = transpose ? out_s.dim : in_s.dim;
  p.out_row = transpose ? in_s.dim : out_s.dim;
  for (int q = 0; q < L.n_skip; ++q) {
    int si = L.skip_in[q], so = L.skip_out[q];
    p.d[q] = 2 * in_s.l[si] + 1;
    if (!transpose) {
      p.in_off[q] = in_s.off[si];
      p.out_off[q] = out_s.off[so];
      p.w[q] = F(c, L.f_skip[q]);
    } else {
      p.in_off[q] = out_s.off[so];
      p.out_off[q] = in_s.off[si];
      p.w[q] = F(c, L.f_skip_t[q]);
    }
    p.tc[q] = tc_find(c, p.w[q]);
  }
  return p;
}

int forward_backward(mace_ctx* c, const mace_system* sys, const mace_outputs* out, int flags,
                     cudaStream_t s) {
  const mace_model_desc& d = c->desc;
  const int64_t N = sys->n_nodes, E = sys->n_edges;
  if (N > c->cap_nodes || E > c->cap_edges)
    return fail(MACE_ERR_BAD_ARG, "system larger than the reserved workspace (call mace_ctx_reserve)");
  if (N <= 0) return fail(MACE_ERR_BAD_ARG, "empty system");
  // active receivers [0, NA) and their edges [0, EA); nodes beyond are senders only
  const int64_t NA = (sys->n_active > 0 && sys->n_active < N) ? sys->n_active : N;
  const int64_t EA = NA < N ? sys->e_active : E;
  if (EA < 0 || EA > E) return fail(MACE_ERR_BAD_ARG, "e_active outside 0 .. n_edges");
  struct Chunk {
    int64_t n0, n1, e0, e1;
  };
  std::vector<Chunk> chunks;
  if (sys->n_chunks <= 1) {
    chunks.push_back({0, NA, 0, EA});
  } else {
    if (!sys->chunk_nodes || !sys->chunk_edges) return fail(MACE_ERR_BAD_ARG, "chunks without boundary arrays");
    const int64_t* cn = sys->chunk_nodes;
    const int64_t* ce = sys->chunk_edges;
    if (cn[0] != 0 || ce[0] != 0 || cn[sys->n_chunks] != NA || ce[sys->n_chunks] != EA)
      return fail(MACE_ERR_BAD_ARG, "chunk boundaries must run from 0 to n_active / e_active (n_nodes / n_edges)");
    for (int k = 0; k < sys->n_chunks; ++k) {
      if (cn[k + 1] < cn[k] || ce[k + 1] < ce[k]) return fail(MACE_ERR_BAD_ARG, "chunk boundaries must not decrease");
      chunks.push_back({cn[k], cn[k + 1], ce[k], ce[k + 1]});
    }
  }
  for (const Chunk& ch : chunks)
    if (ch.e1 - ch.e0 > c->cap_chunk_edges)
      return fail(MACE_ERR_BAD_ARG, "an edge chunk exceeds the reserved chunk capacity (mace_ctx_reserve_chunked)");
  const bool recompute = chunks.size() > 1;
  // When the list is one chunk, the radial-MLP chain (both layers' forwards,
  // each layer's backward once its conv backward is done) runs on a second
  // stream forked from and joined back into `s` with events, so the
  // latency-bound node kernels overlap it (inside a captured graph the fork
  // and join become graph edges).
  const bool fork = !recompute && EA > 0 && !sys->halo && c->dw_layer[0] != nullptr && !c->single_stream;
  if (fork) {
    if (!c->aux) {
      // lowest priority: in eager launches, when both streams have CTAs
      // waiting, the node/conv chain (the step's critical path) is scheduled
      // first.  A replayed graph runs every node at the priority of the
      // stream it is launched into (instantiated without the per-node
      // priority flag, which measured 3 % slower on Si1000).
      int least = 0, greatest = 0;
      MACE_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
      MACE_CUDA_TRY(cudaStreamCreateWithPriority(&c->aux, cudaStreamNonBlocking, least));
    }
    for (cudaEvent_t& e : c->fork_ev)
      if (!e) MACE_CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  }
  cudaStream_t sa = fork ? c->aux : s;
  // Layer 0's radial MLP and conv in two parts each when its tiles exceed one
  // round of MLP CTAs (two per SM): forward, the first round of tiles, then
  // the conv of the receivers whose edges it covers beside the remaining
  // tiles, then the other receivers; backward, the conv of the receivers
  // below the split, then the MLP of those tiles beside the other receivers'
  // conv, then one round of MLP tiles.  The serial MLP work at the start and
  // the end of the step shrinks to about one tile each.
  if (fork && c->sm_count == 0)
    MACE_CUDA_TRY(cudaDeviceGetAttribute(&c->sm_count, cudaDevAttrMultiProcessorCount, c->device));
  const int64_t mlp_round = 2 * (int64_t)c->sm_count;  // MLP tiles resident at once
  const int64_t ntile0 = (EA + WT_TILE - 1) / WT_TILE;
  const bool split0 = fork && ntile0 > mlp_round;
  const int64_t e_split_f = split0 ? mlp_round * WT_TILE : 0;             // forward: first round of tiles
  const int64_t e_split_b = split0 ? (ntile0 - mlp_round) * WT_TILE : 0;  // backward: the last round after
  // events: 0 step start (the second stream's edge front end waits on it);
  // 1+t mlp_fwd(t); 1+T+t conv_bwd(t); 1+2T last mlp_bwd; 2+2T+t dh[t+1] final;
  // 2+3T+t skip_bwd(t) done; 2+4T+t conv_fwd(t) done; 2+5T readouts done;
  // 3+5T first MLP part done; 4+5T first conv_bwd part done
  cudaEvent_t* ev = c->fork_ev;
  const int T = d.num_layers;
  const int C = d.C;
  c->launches = 0;
  c->last_N = N;
  c->last_E = E;
  if (c->prof_on) TRY(prof_fold(c));
  const bool want_grad = (flags & (MACE_WANT_FORCES | MACE_WANT_VIRIAL)) != 0;

  EdgeParams ep{};
  ep.E = E;
  ep.pos = sys->pos;
  ep.cell = sys->cell;
  ep.snd = sys->sender;
  ep.rcv = sys->receiver;
  ep.shifts = sys->shifts;
  ep.max_ell = d.max_ell;
  ep.nb = d.num_bessel;
  ep.r_max = d.r_max;
  ep.poly_p = d.poly_p;
  ep.bessel_w = F(c, d.f_bessel);
  ep.sh_T = F(c, d.f_sh);
  ep.v = c->v;
  ep.Y = c->Y;
  ep.b = c->b;
  ep.dY = c->dY;
  ep.db = c->db;
  ep.dv = c->dv;
  ep.cut = d.envelope_on_weights ? c->cut : nullptr;
  ep.dcut = d.envelope_on_weights ? c->dcut : nullptr;
  ep.virial_part = (flags & MACE_WANT_VIRIAL) ? c->vir_part : nullptr;
  ep.species = sys->species;
  ep.agnesi = d.agnesi;
  if (d.agnesi) {
    ep.ag_q = d.agnesi_q;
    ep.ag_p = d.agnesi_p;
    ep.ag_a = d.agnesi_a;
    ep.ag_radius = F(c, d.f_radius_agnesi);
  }
  ep.zbl = d.zbl;
  if (d.zbl) {
    ep.zbl_p = d.zbl_p;
    ep.zbl_a_exp = d.zbl_a_exp;
    ep.zbl_a_pref = d.zbl_a_prefactor;
    ep.zbl_radius = F(c, d.f_radius_zbl);
    ep.znum = F(c, d.f_znum);
    ep.zbl_dscale = d.scale_shift ? d.scale : 1.0f;
    ep.weight = sys->energy_weight;
  }
  ep.n_dens = 0;
  for (int t = 0; t < d.num_layers; ++t) {
    if (!d.layers[t].density) continue;
    ep.dens_w[ep.n_dens] = F(c, d.layers[t].f_density);
    ep.dD[ep.n_dens] = c->ddens + (int64_t)t * N;
    ++ep.n_dens;
  }
  if (NA < N) {
    // inactive rows are never written by the per-receiver kernels: zero what is read for them
    MACE_CUDA_TRY(cudaMemsetAsync(c->e_layers, 0, sizeof(float) * (size_t)(T + 1) * N, s));
    MACE_CUDA_TRY(cudaMemsetAsync(c->ddens, 0, sizeof(float) * (size_t)T * N, s));
  }
  // In the two-stream step the edge front end (and the per-receiver sums built
  // on it) runs on the second stream ahead of the radial MLP, so that the
  // embedding and layer 0's linear_up run beside it on the main stream instead
  // of waiting for SMs the MLP holds.
  cudaStream_t se = s;
  if (fork) {
    MACE_CUDA_TRY(cudaEventRecord(ev[0], s));
    MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[0], 0));
    se = sa;
  }
  if (E > 0) LAUNCH_ON(se, "edge_fwd", -1, launch_edge_fwd(ep, se));
  if (ep.n_dens > 0 || d.zbl) {
    // per-receiver densities of the density-normalised layers and ZBL pair energies
    NodeSumParams np{};
    np.N = N;
    np.row_ptr = sys->row_ptr;
    np.snd = sys->sender;
    np.species = sys->species;
    np.v = c->v;
    np.b = c->b;
    np.nb = d.num_bessel;
    for (int t = 0; t < d.num_layers; ++t) {
      if (!d.layers[t].density) continue;
      np.dens_w[np.n_dens] = F(c, d.layers[t].f_density);
      np.D[np.n_dens] = c->dens + (int64_t)t * N;
      ++np.n_dens;
    }
    np.zbl = d.zbl;
    np.zbl_p = d.zbl_p;
    np.zbl_a_exp = d.zbl_a_exp;
    np.zbl_a_pref = d.zbl_a_prefactor;
    np.zbl_radius = d.zbl ? F(c, d.f_radius_zbl) : nullptr;
    np.znum = d.zbl ? F(c, d.f_znum) : nullptr;
    np.pair = c->e_layers + (int64_t)d.num_layers * N;
    LAUNCH_ON(se, "node_sums", -1, launch_node_sums(np, se));
  }
  // Layer 0's radial MLP starts as soon as the edge features exist; a later
  // layer's starts once the previous layer's conv is done (below).  The MLP
  // CTAs (two per SM, most of its registers and shared memory) leave no room
  // for conv CTAs, so beside a conv they only delay it; beside the node ops
  // of the previous layer (latency-bound, on few SMs) they cost little.
  if (fork) {
    if (split0) {
      MlpParams ma = mlp_params_tiles(c, 0, 0, e_split_f);
      LAUNCH_ON(sa, "mlp_fwd", 0, launch_mlp_fwd(ma, sa));
      MACE_CUDA_TRY(cudaEventRecord(ev[3 + 5 * T], sa));
      MlpParams mb = mlp_params_tiles(c, 0, e_split_f, EA - e_split_f);
      LAUNCH_ON(sa, "mlp_fwd", 0, launch_mlp_fwd(mb, sa));
    } else {
      MlpParams mp = mlp_params(c, 0, 0, EA);
      LAUNCH_ON(sa, "mlp_fwd", 0, launch_mlp_fwd(mp, sa));
    }
    MACE_CUDA_TRY(cudaEventRecord(ev[1], sa));
  }
  {
    EmbedParams p{N, C, sys->species, F(c, d.f_emb), c->h[0]};
    LAUNCH("embed", -1, launch_embed(p, s));
  }
  const float dscale = d.scale_shift ? d.scale : 1.0f;
  for (int t = 0; t < T; ++t) {
    const mace_layer_desc& L = d.layers[t];
    LayerBufs& B = c->lb[t];
    // skip connection written first; the product linear accumulates onto it
    MACE_CUDA_TRY(cudaMemsetAsync(c->h[t + 1], 0, sizeof(float) * N * L.hid.dim, s));
    {
      // linear_up (h[t] -> up) and, in residual layers, the skip (h[t] -> h[t+1]) in one launch
      LinParams lp{};
      lp.err_flag = c->d_err;
      lp.N = N;
      lp.C = C;
      lp.in = c->h[t];
      lp.in_row = L.in.dim;
      lp.out = B.up;
      lp.out_row = L.in.dim;
      for (int q = 0; q < L.in.n; ++q) {
        int ko = L.in.off[q];
        lp.job[lp.n_jobs++] = make_job(c, 2 * L.in.l[q] + 1, 1, &ko, L.in.off[q], F(c, L.f_up[q]), C, 1.f, 0);
      }
      if (L.residual) {
        SkipParams sp = skip_params(c, t, N, sys->species, false, L.in, L.hid, c->h[t], c->h[t + 1], 0);
        lp.n_jobs += skip_jobs(sp, lp.job + lp.n_jobs);
      }
      LAUNCH("linear_up+skip", t, launch_linear(lp, s));
    }
    if (t == 0 && split0) {
      ConvParams cp = conv_params(c, 0, NA, sys);
      cp.e_split = e_split_f;
      cp.split_part = 1;
      MACE_CUDA_TRY(cudaStreamWaitEvent(s, ev[3 + 5 * T], 0));
      LAUNCH("conv_fwd", 0, launch_conv_fwd(cp, s));
      cp.split_part = 2;
      MACE_CUDA_TRY(cudaStreamWaitEvent(s, ev[1], 0));
      LAUNCH("conv_fwd", 0, launch_conv_fwd(cp, s));
    } else {
      if (fork) MACE_CUDA_TRY(cudaStreamWaitEvent(s, ev[1 + t], 0));
      for (const Chunk& ch : chunks) {
        MlpParams mp = mlp_params(c, t, ch.e0, ch.e1 - ch.e0);
        if (!fork && ch.e1 > ch.e0) LAUNCH("mlp_fwd", t, launch_mlp_fwd(mp, s));
        ConvParams cp = conv_params(c, t, ch.n1, sys);
        cp.n0 = ch.n0;
        cp.e0 = ch.e0;
        LAUNCH("conv_fwd", t, launch_conv_fwd(cp, s));
      }
    }
    if (fork && t + 1 < T) {
      MACE_CUDA_TRY(cudaEventRecord(ev[2 + 4 * T + t], s));
      MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[2 + 4 * T + t], 0));
      MlpParams mp = mlp_params(c, t + 1, 0, EA);
      LAUNCH_ON(sa, "mlp_fwd", t + 1, launch_mlp_fwd(mp, sa));
      MACE_CUDA_TRY(cudaEventRecord(ev[2 + t], sa));
    }
    {
      LinParams lp{};
      lp.err_flag = c->d_err;
      lp.N = N;
      lp.C = C;
      lp.N = NA;
      lp.in = B.A;
      lp.in_row = L.mid.dim;
      lp.out = B.msg;
      lp.out_row = L.inter.dim;
      lp.n_jobs = L.inter.n;
      for (int l = 0; l < L.inter.n; ++l) {
        const mace_lin_group& g = L.lin[l];
        int ko[MACE_MAX_SRC];
        for (int q = 0; q < g.n_src; ++q) ko[q] = L.conv[g.src[q]].off;
        lp.job[l] = make_job(c, 2 * l + 1, g.n_src, ko, L.inter.off[l], F(c, g.f_w), C,
                             L.density ? 1.0f : d.inv_avg_num_neighbors, 0);
      }
      LAUNCH("linear_msg", t, launch_linear(lp, s));
    }
    if (L.density)  // message / (density + 1) instead of / avg_num_neighbors
      LAUNCH("density_scale", t, launch_density_scale(B.msg, L.inter.dim, c->dens + (int64_t)t * N, NA, s));
    const float* sc_in = B.msg;
    if (!L.residual) {
      SkipParams sp = skip_params(c, t, NA, sys->species, false, L.inter, L.inter, B.msg, B.msg2, 0);
      MACE_CUDA_TRY(cudaMemsetAsync(B.msg2, 0, sizeof(float) * N * L.inter.dim, s));
      LAUNCH("skip_fwd", t, launch_skip(sp, s));
      sc_in = B.msg2;
    }
    ScParams scp = sc_params(c, t, NA, sys->species, sc_in, B.B, nullptr, nullptr);
    LAUNCH("sc_fwd", t, launch_sc_fwd(scp, s));
    TRY(run_linear_slots(c, "linear_prod", t, NA, L.hid, L.hid, L.f_prod, B.B, c->h[t + 1], 1, s));
    if (NA < N)  // readout seeds exist for active rows only
      MACE_CUDA_TRY(cudaMemsetAsync(c->dh[t + 1] + NA * L.hid.dim, 0, sizeof(float) * (N - NA) * L.hid.dim, s));
    ReadoutParams rp{};
    rp.N = NA;
    rp.C = C;
    rp.h = c->h[t + 1];
    rp.h_row = L.hid.dim;
    rp.nonlinear = L.readout_nonlinear;
    rp.hidden = L.readout_hidden;
    rp.w1 = F(c, L.f_ro1);
    rp.w2 = L.readout_nonlinear ? F(c, L.f_ro2) : nullptr;
    rp.e = c->e_layers + (int64_t)t * N;
    rp.dh = c->dh[t + 1];
    rp.dscale = dscale;
    rp.weight = sys->energy_weight;
    LAUNCH("readout", t, launch_readout(rp, s));
    if (sys->halo_exchange && t + 1 < T) {
      TRY(launch(c, "halo_features", t, s, [&]() { return halo_features(sys->halo_exchange, c->h[t + 1], L.hid.dim, s); }));
    } else if (sys->halo && t + 1 < T) {
      if (sys->halo(sys->halo_user, MACE_HALO_FEATURES, t, c->h[t + 1], L.hid.dim, s) != 0)
        return fail(MACE_ERR_NCCL, "halo exchange of node features failed");
    }
  }
  {
    EnergyParams p{};
    p.N = N;
    p.num_graphs = sys->num_graphs;
    p.T = T;
    p.species = sys->species;
    p.graph_ptr = sys->graph_ptr;
    p.e0 = F(c, d.f_e0);
    p.e_layers = c->e_layers;
    if (d.zbl) p.T = T + 1;  // the pair energies are one more (scaled) interaction term
    p.scale_shift = d.scale_shift;
    p.scale = d.scale;
    p.shift = d.shift;
    p.node_energy = out ? out->node_energy : nullptr;
    p.energy = out ? out->energy : nullptr;
    p.weight = sys->energy_weight;
    if (fork && want_grad) {
      // nothing in the backward reads the energies: the assembly runs on the
      // second stream (joined with it at the end of the step)
      MACE_CUDA_TRY(cudaEventRecord(ev[2 + 5 * T], s));
      MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[2 + 5 * T], 0));
      LAUNCH_ON(sa, "energy", -1, launch_energy(p, sa));
    } else {
      LAUNCH("energy", -1, launch_energy(p, s));
    }
  }
  if (!want_grad) return MACE_OK;

  if (E > 0) {
    MACE_CUDA_TRY(cudaMemsetAsync(c->dY, 0, sizeof(float) * E * 16, s));
    MACE_CUDA_TRY(cudaMemsetAsync(c->db, 0, sizeof(float) * E * d.num_bessel, s));
    if (d.envelope_on_weights) MACE_CUDA_TRY(cudaMemsetAsync(c->dcut, 0, sizeof(float) * E, s));
  }
  for (int t = T - 1; t >= 0; --t) {
    const mace_layer_desc& L = d.layers[t];
    LayerBufs& B = c->lb[t];
    // the residual skip's gradient (dh[t+1] -> dh[t]) only needs dh[t+1]: it
    // accumulates into dh[t] first (same order with and without the fork), on
    // the second stream overlapping this layer's backward and joined before
    // linear_up_bwd accumulates into dh[t]
    const bool early_skip = t > 0 && L.residual;
    if (early_skip) {
      if (fork) {
        MACE_CUDA_TRY(cudaEventRecord(ev[2 + 2 * T + t], s));
        MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[2 + 2 * T + t], 0));
      }
      SkipParams sp = skip_params(c, t, NA, sys->species, true, L.in, L.hid, c->dh[t + 1], c->dh[t], 1);
      LAUNCH_ON(sa, "skip_bwd", t, launch_skip(sp, sa));
      if (fork) MACE_CUDA_TRY(cudaEventRecord(ev[2 + 3 * T + t], sa));
    }
    TRY(run_linear_slots(c, "linear_prod_bwd", t, NA, L.hid, L.hid, L.f_prod_t, c->dh[t + 1], B.dB, 0, s));
    float* dsc_in = B.dmsg;
    ScParams scp = sc_params(c, t, NA, sys->species, L.residual ? B.msg : B.msg2, nullptr, B.dB,
                             L.residual ? B.dmsg : B.dmsg2);
    LAUNCH("sc_bwd", t, launch_sc_bwd(scp, s));
    if (!L.residual) {
      MACE_CUDA_TRY(cudaMemsetAsync(B.dmsg, 0, sizeof(float) * N * L.inter.dim, s));
      SkipParams sp = skip_params(c, t, NA, sys->species, true, L.inter, L.inter, B.dmsg2, B.dmsg, 1);
      LAUNCH("skip_bwd", t, launch_skip(sp, s));
    }
    if (L.density)  // through message = linear(A) / (D + 1): dD, and dmsg / (D + 1)
      LAUNCH("density_bwd", t, launch_density_bwd(B.msg, B.dmsg, L.inter.dim, c->dens + (int64_t)t * N,
                                                  c->ddens + (int64_t)t * N, NA, s));
    {
      // dA[mid slot k] = inv_avg * dmsg[inter slot l_k] @ W_l^T (block q of the concat-K)
      LinParams lp{};
      lp.err_flag = c->d_err;
      lp.N = N;
      lp.C = C;
      lp.N = NA;
      lp.in = dsc_in;
      lp.in_row = L.inter.dim;
      lp.out = B.dA;
      lp.out_row = L.mid.dim;
      lp.n_jobs = 0;
      for (int l = 0; l < L.inter.n; ++l) {
        const mace_lin_group& g = L.lin[l];
        for (int q = 0; q < g.n_src; ++q) {
          int ko = L.inter.off[l];
          lp.job[lp.n_jobs++] = make_job(c, 2 * l + 1, 1, &ko, L.conv[g.src[q]].off, F(c, g.f_wt) + q * C,
                                         g.n_src * C, L.density ? 1.0f : d.inv_avg_num_neighbors, 0);
        }
      }
      LAUNCH("linear_msg_bwd", t, launch_linear(lp, s));
      if (NA < N)  // receivers beyond n_active carry no gradient
        MACE_CUDA_TRY(cudaMemsetAsync(B.dA + NA * L.mid.dim, 0, sizeof(float) * (N - NA) * L.mid.dim, s));
    }
    bool need_gather = false;
    for (const Chunk& ch : chunks) {
      MlpParams mp = mlp_params(c, t, ch.e0, ch.e1 - ch.e0);
      // several chunks share the weight buffers: recompute this chunk's radial weights
      if (recompute && ch.e1 > ch.e0) LAUNCH("mlp_fwd", t, launch_mlp_fwd(mp, s));
      ConvParams cp = conv_params(c, t, ch.n1, sys);
      cp.n0 = ch.n0;
      cp.e0 = ch.e0;
      bool gather = false;
      cp.n_active = NA < N ? NA : 0;
      if (t == 0 && split0) {
        // receivers whose first edge is below the split, then those tiles' MLP
        // backward beside the other receivers' conv, then the last round of tiles
        cp.e_split = e_split_b;
        cp.split_first = 1;
        cp.split_part = 1;
        LAUNCH("conv_bwd", 0, launch_conv_bwd(cp, s, &gather));
        MACE_CUDA_TRY(cudaEventRecord(ev[4 + 5 * T], s));
        MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[4 + 5 * T], 0));
        MlpParams ma = mlp_params_tiles(c, 0, 0, e_split_b);
        LAUNCH_ON(sa, "mlp_bwd", 0, launch_mlp_bwd(ma, sa));
        bool gather2 = false;
        cp.split_part = 2;
        LAUNCH("conv_bwd", 0, launch_conv_bwd(cp, s, &gather2));
        need_gather = need_gather || gather || gather2;
        MACE_CUDA_TRY(cudaEventRecord(ev[1 + T], s));
        MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[1 + T], 0));
        MlpParams mb = mlp_params_tiles(c, 0, e_split_b, EA - e_split_b);
        LAUNCH_ON(sa, "mlp_bwd", 0, launch_mlp_bwd(mb, sa));
        continue;
      }
      LAUNCH("conv_bwd", t, launch_conv_bwd(cp, s, &gather));
      if (NA < N && t > 0 && !gather)
        return fail(MACE_ERR_UNSUPPORTED, "n_active needs the per-edge sender terms of the conv backward (one radial "
                                          "chunk and a layer signature of conv_sig.cu)");
      need_gather = need_gather || gather;
      if (fork) {
        MACE_CUDA_TRY(cudaEventRecord(ev[1 + T + t], s));
        MACE_CUDA_TRY(cudaStreamWaitEvent(sa, ev[1 + T + t], 0));
        LAUNCH_ON(sa, "mlp_bwd", t, launch_mlp_bwd(mp, sa));
      } else if (ch.e1 > ch.e0) {
        LAUNCH("mlp_bwd", t, launch_mlp_bwd(mp, s));
      }
    }
    if (need_gather) {
      // the sender-side terms of every chunk's edges are in place: sum them per node
      ConvParams cp = conv_params(c, t, N, sys);
      cp.n_active = NA < N ? NA : 0;
      LAUNCH("dup_gather", t, launch_dup_gather(cp, s));
    }
    if (t > 0) {
      // dh[t] holds the readout seed of layer t-1
      if (early_skip && fork) MACE_CUDA_TRY(cudaStreamWaitEvent(s, ev[2 + 3 * T + t], 0));
      TRY(run_linear_slots(c, "linear_up_bwd", t, N, L.in, L.in, L.f_up_t, B.dup, c->dh[t], 1, s));
      // dh[t]: gradient w.r.t. the features layer t - 1 produced
      if (sys->halo_exchange) {
        TRY(launch(c, "halo_gradients", t - 1, s,
                   [&]() { return halo_gradients(sys->halo_exchange, c->dh[t], L.in.dim, s); }));
      } else if (sys->halo && sys->halo(sys->halo_user, MACE_HALO_GRADIENTS, t - 1, c->dh[t], L.in.dim, s) != 0) {
        return fail(MACE_ERR_NCCL, "halo reduction of feature gradients failed");
      }
    }
  }
  if (fork) {  // join: every MLP backward has accumulated into db
    MACE_CUDA_TRY(cudaEventRecord(ev[1 + 2 * T], sa));
    MACE_CUDA_TRY(cudaStreamWaitEvent(s, ev[1 + 2 * T], 0));
  }
  int n_blocks = (int)((E + 255) / 256);
  if (E > 0) LAUNCH("edge_bwd", -1, launch_edge_bwd(ep, &n_blocks, s));
  if (out && out->forces) {
    if (E > 0) {
      ForceParams fp{N, sys->row_ptr, sys->sender, sys->receiver, sys->rev, c->dv, out->forces, c->d_err};
      LAUNCH("forces", -1, launch_forces(fp, s));
    } else {
      MACE_CUDA_TRY(cudaMemsetAsync(out->forces, 0, sizeof(float) * 3 * N, s));
    }
  }
  if ((flags & MACE_WANT_VIRIAL) && out && out->virial) {
    if (E > 0) {
      LAUNCH("virial", -1, launch_virial_reduce(c->vir_part, n_blocks, out->virial, s));
    } else {
      MACE_CUDA_TRY(cudaMemsetAsync(out->virial, 0, sizeof(double) * 9, s));
    }
  }
  return MACE_OK;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
namespace {

// Cell-list geometry for one graph of n atoms (p.reach and the inverse cell set
// when any axis is periodic; wraps computed): bins per axis at least one reach
// wide, at least 3 along periodic axes (else all pairs), over the wrapped
// [0, 1) range along periodic axes and the atoms' range along open ones
// (fractional with a cell, Cartesian without).
int nl_choose_mode(mace_ctx* c, NlParams& p, bool any_pbc, int32_t num_graphs, int64_t n, cudaStream_t s) {
  // all pairs are cheaper for small graphs; MACE_B200_NL_CELL_MIN overrides the 2048-atom threshold
  const char* env = std::getenv("MACE_B200_NL_CELL_MIN");
  const int64_t cl_min = env ? std::atoll(env) : 2048;
  p.mode = 0;
  if (num_graphs != 1 || n < cl_min) return MACE_OK;
  p.use_frac = any_pbc ? 1 : 0;
  p.mode = 1;  // bin_space reads use_frac; set before the bounding box
  TRY(launch_nl_bbox(p, c->nl_bbox, s));
  double bb[6];
  MACE_CUDA_TRY(cudaMemcpyAsync(bb, c->nl_bbox, sizeof(bb), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  p.mode = 0;
  int64_t nb[3];
  double ext[3];
  for (int d = 0; d < 3; ++d) {
    const double unit = any_pbc ? p.reach[d] : p.r_cut;  // one cutoff in bin coordinates
    if (p.pbc[d]) {
      nb[d] = (int64_t)std::floor(1.0 / unit);
      if (nb[d] < 3) return MACE_OK;
      ext[d] = 1.0;
    } else {
      ext[d] = bb[3 + d] - bb[d];
      nb[d] = (int64_t)std::floor(ext[d] / unit);
      if (nb[d] < 1) nb[d] = 1;
      p.origin[d] = bb[d];
    }
  }
  // at most nl_bin_cap bins: merge bins along the longest axis (bins only widen)
  while (nb[0] * nb[1] * nb[2] > c->nl_bin_cap) {
    int d = 0;
    for (int q = 1; q < 3; ++q) d = nb[q] > nb[d] ? q : d;
    const int64_t floor_nb = p.pbc[d] ? 3 : 1;
    if (nb[d] <= floor_nb) return MACE_OK;
    nb[d] = (nb[d] * 3) / 4 > floor_nb ? (nb[d] * 3) / 4 : floor_nb;
  }
  for (int d = 0; d < 3; ++d) {
    p.nbin[d] = (int)nb[d];
    p.inv_binw[d] = (!p.pbc[d] && ext[d] > 0.0) ? (double)nb[d] / ext[d] : 0.0;
  }
  p.mode = 1;
  p.atom_bin = c->nl_atom_bin;
  p.bin_start = c->nl_bin_start;
  p.bin_fill = c->nl_bin_fill;
  p.bin_atoms = c->nl_bin_atoms;
  return MACE_OK;
}

int nl_build(mace_ctx* c, const double* pos, const double* cell, const int32_t* pbc, const int32_t* graph_ptr,
             int32_t num_graphs, int64_t n, double r_cut, int32_t* sender, int32_t* receiver, int32_t* shifts,
             int32_t* row_ptr, int32_t* rev, int64_t capacity, int64_t* n_edges, bool allow_cells,
             cudaStream_t s) {
  NlParams p{};
  p.n = n;
  p.pos = pos;
  p.cell = cell;
  p.r_cut = r_cut;
  p.graph_ptr = graph_ptr;
  p.num_graphs = num_graphs;
  bool any_pbc = false;
  for (int d = 0; d < 3; ++d) {
    p.pbc[d] = pbc[d] ? 1 : 0;
    any_pbc |= pbc[d] != 0;
  }
  double hc[9] = {0}, inv[9] = {0};
  if (any_pbc) {
    if (!cell) return fail(MACE_ERR_BAD_ARG, "periodic system without a cell");
    MACE_CUDA_TRY(cudaMemcpyAsync(hc, cell, sizeof(hc), cudaMemcpyDeviceToHost, s));
    MACE_CUDA_TRY(cudaStreamSynchronize(s));
    double det = hc[0] * (hc[4] * hc[8] - hc[5] * hc[7]) - hc[1] * (hc[3] * hc[8] - hc[5] * hc[6]) +
                 hc[2] * (hc[3] * hc[7] - hc[4] * hc[6]);
    if (!(std::fabs(det) > 1e-12)) return fail(MACE_ERR_BAD_ARG, "periodic cell is singular");
    inv[0] = (hc[4] * hc[8] - hc[5] * hc[7]) / det;
    inv[1] = (hc[2] * hc[7] - hc[1] * hc[8]) / det;
    inv[2] = (hc[1] * hc[5] - hc[2] * hc[4]) / det;
    inv[3] = (hc[5] * hc[6] - hc[3] * hc[8]) / det;
    inv[4] = (hc[0] * hc[8] - hc[2] * hc[6]) / det;
    inv[5] = (hc[2] * hc[3] - hc[0] * hc[5]) / det;
    inv[6] = (hc[3] * hc[7] - hc[4] * hc[6]) / det;
    inv[7] = (hc[1] * hc[6] - hc[0] * hc[7]) / det;
    inv[8] = (hc[0] * hc[4] - hc[1] * hc[3]) / det;
    const double vol = std::fabs(det);
    for (int d = 0; d < 3; ++d) {
      const double* a = hc + 3 * ((d + 1) % 3);
      const double* b = hc + 3 * ((d + 2) % 3);
      double cx = a[1] * b[2] - a[2] * b[1], cy = a[2] * b[0] - a[0] * b[2], cz = a[0] * b[1] - a[1] * b[0];
      double h = vol / std::sqrt(cx * cx + cy * cy + cz * cz);
      p.reach[d] = r_cut / h * (1.0 + 1e-9) + 1e-9;
    }
  }
  MACE_CUDA_TRY(cudaMemcpyAsync(c->nl_inv, inv, sizeof(inv), cudaMemcpyHostToDevice, s));
  p.inv_cell = c->nl_inv;
  p.count = c->nl_count;
  p.row_ptr = row_ptr;
  p.snd = sender;
  p.rcv = receiver;
  p.shifts = shifts;
  p.rev = rev;
  p.err_flag = c->d_err;
  p.node_graph = c->nl_graph;
  p.wrap = c->nl_wrap;
  TRY(launch_nl_prep(p, c->nl_graph, c->nl_wrap, s));
  if (allow_cells) TRY(nl_choose_mode(c, p, any_pbc, num_graphs, n, s));
  if (p.mode) {
    TRY(launch_nl_bins(p, c->scan_tmp, c->scan_bytes, s));
    TRY(launch_nl_cl_count(p, s));
  } else {
    TRY(launch_nl_count(p, s));
  }
  MACE_CUDA_TRY(cudaMemsetAsync(c->nl_count + n, 0, sizeof(int32_t), s));
  TRY(scan_counts(c->nl_count, row_ptr, n, c->scan_tmp, c->scan_bytes, s));
  int32_t total = 0;
  MACE_CUDA_TRY(cudaMemcpyAsync(&total, row_ptr + n, sizeof(int32_t), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  *n_edges = total;
  if (total > capacity) return fail(MACE_ERR_NL_OVERFLOW, "edge capacity too small");
  if (total > 0 && (!sender || !receiver || !shifts || !rev)) return fail(MACE_ERR_BAD_ARG, "null edge output");
  MACE_CUDA_TRY(cudaMemsetAsync(c->d_err, 0, sizeof(int), s));
  if (p.mode) {
    if (total > c->nl_keys_cap) {
      if (c->nl_keys) cudaFree(c->nl_keys);
      c->nl_keys = nullptr;
      c->nl_keys_cap = 0;
      MACE_CUDA_TRY(cudaMalloc(&c->nl_keys, sizeof(unsigned long long) * (size_t)(total > 0 ? total : 1)));
      c->nl_keys_cap = total;
    }
    p.keys = c->nl_keys;
    TRY(launch_nl_cl_fill(p, s));
  } else {
    TRY(launch_nl_fill(p, s));
  }
  int err = 0;
  MACE_CUDA_TRY(cudaMemcpyAsync(&err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  if (err == NL_ERR_SHIFT)  // a shift beyond the cell-list key range: all pairs instead
    return nl_build(c, pos, cell, pbc, graph_ptr, num_graphs, n, r_cut, sender, receiver, shifts, row_ptr, rev,
                    capacity, n_edges, false, s);
  TRY(launch_nl_rev(p, total, s));
  MACE_CUDA_TRY(cudaMemcpyAsync(&err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, s));
  MACE_CUDA_TRY(cudaStreamSynchronize(s));
  if (err) return fail(MACE_ERR_EDGES, "neighbour list is not closed under edge reversal");
  return MACE_OK;
}

}  // namespace

namespace mace {
void ctx_drop_graph(mace_ctx* c) {
  DeviceGuard g(c->device);
  drop_graph(c);
}
}  // namespace mace

extern "C" {

int mace_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return MACE_ERR_BAD_ARG;
  std::snprintf(buf, len, "%s", g_last_error.c_str());
  return MACE_OK;
}

// tensor-core images of every node-linear weight the step uses (one
// allocation, made once: the weights never change)
int tc_prepare(mace_ctx* c) {
  const mace_model_desc& d = c->desc;
  const int C = d.C;
  struct Want {
    const float* w;
    int K, ldb, Z;
    int64_t zstride;
  };
  std::vector<Want> want;
  for (int t = 0; t < d.num_layers; ++t) {
    const mace_layer_desc& L = d.layers[t];
    for (int q = 0; q < L.in.n; ++q) {
      want.push_back({F(c, L.f_up[q]), C, C, 1, 0});
      want.push_back({F(c, L.f_up_t[q]), C, C, 1, 0});
    }
    for (int q = 0; q < L.hid.n; ++q) {
      want.push_back({F(c, L.f_prod[q]), C, C, 1, 0});
      want.push_back({F(c, L.f_prod_t[q]), C, C, 1, 0});
    }
    for (int l = 0; l < L.inter.n; ++l) {
      const mace_lin_group& g = L.lin[l];
      want.push_back({F(c, g.f_w), g.n_src * C, C, 1, 0});
      for (int q = 0; q < g.n_src; ++q) want.push_back({F(c, g.f_wt) + q * C, C, g.n_src * C, 1, 0});
    }
    for (int q = 0; q < L.n_skip; ++q) {
      want.push_back({F(c, L.f_skip[q]), C, C, d.num_elements, (int64_t)C * C});
      want.push_back({F(c, L.f_skip_t[q]), C, C, d.num_elements, (int64_t)C * C});
    }
  }
  int64_t total = 0;
  for (const Want& x : want) total += tc_image_floats(x.K, C, x.Z);
  if (total == 0) return MACE_OK;
  MACE_CUDA_TRY(cudaMalloc(&c->tc_images, sizeof(float) * total));
  int64_t off = 0;
  for (const Want& x : want) {
    if (tc_find(c, x.w)) continue;
    float* img = c->tc_images + off;
    TRY(launch_tc_image(x.w, x.K, x.ldb, C, x.Z, x.zstride, img, 0));
    c->tc_index.push_back({x.w, img});
    off += tc_image_floats(x.K, C, x.Z);
  }
  MACE_CUDA_TRY(cudaStreamSynchronize(0));
  return MACE_OK;
}

int mace_ctx_create(const mace_model_desc* desc, int device, mace_ctx** out) {
  if (!desc || !out) return fail(MACE_ERR_BAD_ARG, "null argument");
  if (desc->abi_version != MACE_ABI_VERSION) return fail(MACE_ERR_BAD_ARG, "model description ABI version mismatch");
  if (desc->num_layers < 1 || desc->num_layers > MACE_MAX_LAYERS)
    return fail(MACE_ERR_UNSUPPORTED, "number of interaction layers out of range");
  if (desc->max_ell < 0 || desc->max_ell > 3) return fail(MACE_ERR_UNSUPPORTED, "max_ell must be <= 3");
  if (desc->C % 32 != 0 || desc->C > 128) return fail(MACE_ERR_UNSUPPORTED, "channels must be 32, 64, 96 or 128");
  if (desc->envelope_on_weights) {
    for (int t = 0; t < desc->num_layers; ++t)
      if (desc->layers[t].density)
        return fail(MACE_ERR_UNSUPPORTED, "envelope_on_weights with density-normalised layers is not supported");
  }
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(MACE_ERR_CUDA, "no such CUDA device");
  DeviceGuard g(device);
  mace_ctx* c = new mace_ctx();
  c->device = device;
  c->desc = *desc;
  cudaError_t e1 = cudaMalloc(&c->d_floats, sizeof(float) * (desc->n_floats > 0 ? desc->n_floats : 1));
  cudaError_t e2 = cudaMalloc(&c->d_ints, sizeof(int32_t) * (desc->n_ints > 0 ? desc->n_ints : 1));
  if (e1 != cudaSuccess || e2 != cudaSuccess) {
    cudaFree(c->d_floats);
    cudaFree(c->d_ints);
    delete c;
    return fail(MACE_ERR_CUDA, "model table allocation failed");
  }
  cudaMemcpy(c->d_floats, desc->floats, sizeof(float) * desc->n_floats, cudaMemcpyHostToDevice);
  cudaError_t e3 = cudaMemcpy(c->d_ints, desc->ints, sizeof(int32_t) * desc->n_ints, cudaMemcpyHostToDevice);
  if (e3 != cudaSuccess) {
    cudaFree(c->d_floats);
    cudaFree(c->d_ints);
    delete c;
    return fail(MACE_ERR_CUDA, std::string("model table upload: ") + cudaGetErrorString(e3));
  }
  c->desc.floats = nullptr;
  c->desc.ints = nullptr;
  const char* env = std::getenv("MACE_B200_MLP_CUDA_CORES");
  c->mlp_cuda_cores = env && env[0] == '1';
  const char* senv = std::getenv("MACE_B200_SINGLE_STREAM");
  c->single_stream = senv && senv[0] == '1';
  const char* lenv = std::getenv("MACE_B200_LINEAR_CUDA_CORES");
  if (!(lenv && lenv[0] == '1')) {
    const int rc = tc_prepare(c);
    if (rc) {
      cudaFree(c->tc_images);
      cudaFree(c->d_floats);
      cudaFree(c->d_ints);
      delete c;
      return rc;
    }
  }
  *out = c;
  return MACE_OK;
}

int mace_ctx_destroy(mace_ctx* c) {
  if (!c) return MACE_OK;
  DeviceGuard g(c->device);
  free_ws(c);
  if (c->ev[0])
    for (int i = 0; i < 2 * mace_ctx::PROF_MAX; ++i) cudaEventDestroy(c->ev[i]);
  drop_graph(c);
  if (c->cap_stream) cudaStreamDestroy(c->cap_stream);
  if (c->aux) cudaStreamDestroy(c->aux);
  for (cudaEvent_t e : c->fork_ev)
    if (e) cudaEventDestroy(e);
  cudaFree(c->tc_images);
  cudaFree(c->d_floats);
  cudaFree(c->d_ints);
  delete c;
  return MACE_OK;
}

int mace_ctx_reserve_chunked(mace_ctx* c, int64_t max_nodes, int64_t max_edges, int64_t max_chunk_edges) {
  if (!c || max_nodes < 0 || max_edges < 0 || max_chunk_edges < 0)
    return fail(MACE_ERR_BAD_ARG, "bad reserve arguments");
  if (max_chunk_edges > max_edges) max_chunk_edges = max_edges;
  if (max_nodes <= c->cap_nodes && max_edges <= c->cap_edges && max_chunk_edges <= c->cap_chunk_edges &&
      c->cap_nodes > 0)
    return MACE_OK;
  DeviceGuard g(c->device);
  const int64_t N = max_nodes > c->cap_nodes ? max_nodes : c->cap_nodes;
  const int64_t E = max_edges > c->cap_edges ? max_edges : c->cap_edges;
  const int64_t EC = max_chunk_edges > c->cap_chunk_edges ? max_chunk_edges : c->cap_chunk_edges;
  MACE_CUDA_TRY(cudaDeviceSynchronize());
  return reserve(c, N < 1 ? 1 : N, E < 1 ? 1 : E, EC < 1 ? 1 : EC);
}

int mace_ctx_reserve(mace_ctx* c, int64_t max_nodes, int64_t max_edges) {
  return mace_ctx_reserve_chunked(c, max_nodes, max_edges, max_edges);
}

int mace_ctx_workspace_bytes(const mace_ctx* c, int64_t* bytes) {
  if (!c || !bytes) return fail(MACE_ERR_BAD_ARG, "null argument");
  *bytes = c->ws_bytes;
  return MACE_OK;
}

int mace_nl_build(mace_ctx* c, const double* pos, const double* cell, const int32_t* pbc,
                  const int32_t* graph_ptr, int32_t num_graphs, int64_t n, double r_cut,
                  int32_t* sender, int32_t* receiver, int32_t* shifts, int32_t* row_ptr, int32_t* rev,
                  int64_t capacity, int64_t* n_edges, void* stream) {
  if (!c || !pos || !pbc || !graph_ptr || !n_edges || !row_ptr) return fail(MACE_ERR_BAD_ARG, "null argument");
  if (n <= 0 || num_graphs <= 0 || !(r_cut > 0)) return fail(MACE_ERR_BAD_ARG, "bad sizes or cutoff");
  if (n > c->cap_nodes) return fail(MACE_ERR_BAD_ARG, "more atoms than reserved (call mace_ctx_reserve)");
  DeviceGuard g(c->device);
  const char* env = std::getenv("MACE_B200_NL_ALL_PAIRS");
  const bool allow_cells = !(env && env[0] == '1');
  return nl_build(c, pos, cell, pbc, graph_ptr, num_graphs, n, r_cut, sender, receiver, shifts, row_ptr, rev,
                  capacity, n_edges, allow_cells, reinterpret_cast<cudaStream_t>(stream));
}

int mace_forward_backward(mace_ctx* c, const mace_system* sys, const mace_outputs* out, int32_t flags,
                          void* stream) {
  if (!c || !sys) return fail(MACE_ERR_BAD_ARG, "null argument");
  if (sys->num_graphs < 1 || !sys->graph_ptr || !sys->species || !sys->pos || !sys->row_ptr)
    return fail(MACE_ERR_BAD_ARG, "incomplete system description");
  if (sys->n_edges > 0 && (!sys->sender || !sys->receiver || !sys->shifts || !sys->rev))
    return fail(MACE_ERR_BAD_ARG, "edges without sender/receiver/shift/rev arrays");
  DeviceGuard g(c->device);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int base_flags = flags & ~MACE_USE_GRAPH;
  if (!(flags & MACE_USE_GRAPH) || sys->halo) return forward_backward(c, sys, out, base_flags, s);
  mace_outputs o{};
  if (out) o = *out;
  std::vector<int64_t> chunk_key;
  if (sys->n_chunks > 1 && sys->chunk_nodes && sys->chunk_edges) {
    chunk_key.assign(sys->chunk_nodes, sys->chunk_nodes + sys->n_chunks + 1);
    chunk_key.insert(chunk_key.end(), sys->chunk_edges, sys->chunk_edges + sys->n_chunks + 1);
  }
  if (c->prof_on) TRY(prof_fold(c));  // the previous replay's events
  const bool same = c->gexec && c->g_flags == base_flags && c->g_prof == c->prof_on &&
                    std::memcmp(&c->g_sys, sys, sizeof(mace_system)) == 0 &&
                    std::memcmp(&c->g_out, &o, sizeof(mace_outputs)) == 0 && c->g_chunks == chunk_key &&
                    c->g_halo_version == halo_version(sys->halo_exchange);
  if (!same) {
    drop_graph(c);
    if (!c->cap_stream) {
      // highest priority; the captured nodes record it, but the graph is
      // instantiated without per-node priorities (see the second stream above)
      int least = 0, greatest = 0;
      MACE_CUDA_TRY(cudaDeviceGetStreamPriorityRange(&least, &greatest));
      MACE_CUDA_TRY(cudaStreamCreateWithPriority(&c->cap_stream, cudaStreamNonBlocking, greatest));
    }
    // order the capture after the caller's prior work (workspace reuse)
    MACE_CUDA_TRY(cudaStreamSynchronize(s));
    MACE_CUDA_TRY(cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal));
    int rc = forward_backward(c, sys, out, base_flags, c->cap_stream);
    cudaGraph_t graph = nullptr;
    cudaError_t ce = cudaStreamEndCapture(c->cap_stream, &graph);
    if (rc) {
      if (graph) cudaGraphDestroy(graph);
      return rc;
    }
    if (ce != cudaSuccess) return fail(MACE_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&c->gexec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess) {
      c->gexec = nullptr;
      return fail(MACE_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(ce));
    }
    c->g_sys = *sys;
    c->g_out = o;
    c->g_flags = base_flags;
    c->g_prof = c->prof_on;
    c->g_prof_n = c->prof_n;
    c->g_chunks = chunk_key;
    c->g_launches = c->launches;
    c->g_halo_version = halo_version(sys->halo_exchange);
    c->g_halo = sys->halo_exchange;
    halo_attach_graph(c->g_halo, c);
  }
  MACE_CUDA_TRY(cudaGraphLaunch(c->gexec, s));
  c->launches = c->g_launches;
  if (c->prof_on) c->prof_n = c->g_prof_n;
  c->last_N = sys->n_nodes;
  c->last_E = sys->n_edges;
  return MACE_OK;
}

int mace_debug_buffer(mace_ctx* c, int32_t id, const float** ptr, int64_t* len) {
  if (!c || !ptr || !len) return fail(MACE_ERR_BAD_ARG, "null argument");
  const int64_t N = c->last_N, E = c->last_E;
  const int layer = id / 16, stage = id % 16;
  *ptr = nullptr;
  *len = 0;
  if (layer == 15) {
    switch (stage) {
      case 0: *ptr = c->v; *len = E * 3; break;
      case 1: *ptr = c->Y; *len = E * 16; break;
      case 2: *ptr = c->b; *len = E * c->desc.num_bessel; break;
      case 3: *ptr = c->dY; *len = E * 16; break;
      case 4: *ptr = c->db; *len = E * c->desc.num_bessel; break;
      case 5: *ptr = c->dv; *len = E * 3; break;
      case 6: *ptr = c->h[0]; *len = N * c->h_row[0]; break;
      case 7: *ptr = c->e_layers; *len = N * (c->desc.num_layers + (c->desc.zbl ? 1 : 0)); break;
      case 8: *ptr = c->dens; *len = N * c->desc.num_layers; break;
      default: return fail(MACE_ERR_BAD_ARG, "unknown debug buffer");
    }
    return MACE_OK;
  }
  if (layer < 0 || layer >= c->desc.num_layers) return fail(MACE_ERR_BAD_ARG, "unknown debug layer");
  const mace_layer_desc& L = c->desc.layers[layer];
  const LayerBufs& B = c->lb[layer];
  switch (stage) {
    case 0: *ptr = B.up; *len = N * L.in.dim; break;
    case 1: *ptr = B.w; *len = wt_floats(E < c->cap_chunk_edges ? E : c->cap_chunk_edges, L.wnumel); break;
    case 2: *ptr = B.A; *len = N * L.mid.dim; break;
    case 3: *ptr = B.msg; *len = N * L.inter.dim; break;
    case 4: *ptr = B.B; *len = N * L.hid.dim; break;
    case 5: *ptr = c->h[layer + 1]; *len = N * L.hid.dim; break;
    case 6: *ptr = c->dh[layer + 1]; *len = N * L.hid.dim; break;
    case 7: *ptr = B.dB; *len = N * L.hid.dim; break;
    case 8: *ptr = B.dmsg; *len = N * L.inter.dim; break;
    case 9: *ptr = B.dA; *len = N * L.mid.dim; break;
    case 10: *ptr = B.dup; *len = N * L.in.dim; break;
    case 11: *ptr = B.act; *len = E * (L.n_mlp - 1) * L.mlp_w[1]; break;
    case 12: *ptr = c->dh[layer]; *len = N * c->h_row[layer]; break;
    case 13: *ptr = B.msg2; *len = B.msg2 ? N * L.inter.dim : 0; break;
    default: return fail(MACE_ERR_BAD_ARG, "unknown debug stage");
  }
  return MACE_OK;
}

int mace_profile_enable(mace_ctx* c, int32_t enable) {
  if (!c) return fail(MACE_ERR_BAD_ARG, "null argument");
  DeviceGuard g(c->device);
  if (enable && !c->ev[0]) {
    for (int i = 0; i < 2 * mace_ctx::PROF_MAX; ++i) MACE_CUDA_TRY(cudaEventCreate(&c->ev[i]));
  }
  if (c->prof_on && c->prof_n) TRY(prof_fold(c));
  c->prof_on = enable != 0;
  c->prof_n = 0;
  c->prof_acc.clear();
  return MACE_OK;
}

int mace_profile_read(mace_ctx* c, int32_t max_entries, char* names, int32_t* layers, int32_t* counts,
                      double* total_ms, int32_t* n_entries) {
  if (!c || !n_entries) return fail(MACE_ERR_BAD_ARG, "null argument");
  DeviceGuard g(c->device);
  TRY(prof_fold(c));
  int n = 0;
  for (const auto& a : c->prof_acc) {
    if (n >= max_entries) break;
    if (names) std::snprintf(names + 32 * n, 32, "%s", a.name.c_str());
    if (layers) layers[n] = a.layer;
    if (counts) counts[n] = a.count;
    if (total_ms) total_ms[n] = a.ms;
    ++n;
  }
  *n_entries = n;
  c->prof_acc.clear();
  return MACE_OK;
}

int mace_profile_timeline(mace_ctx* c, int32_t max_entries, char* names, int32_t* layers, int32_t* streams,
                          float* start_ms, float* end_ms, int32_t* n_entries) {
  if (!c || !n_entries) return fail(MACE_ERR_BAD_ARG, "null argument");
  DeviceGuard g(c->device);
  TRY(prof_fold(c));
  int n = 0;
  for (const auto& a : c->prof_last) {
    if (n >= max_entries) break;
    if (names) std::snprintf(names + 32 * n, 32, "%s", a.name.c_str());
    if (layers) layers[n] = a.layer;
    if (streams) streams[n] = a.stream;
    if (start_ms) start_ms[n] = a.t0;
    if (end_ms) end_ms[n] = a.t1;
    ++n;
  }
  *n_entries = n;
  return MACE_OK;
}

int mace_last_launch_count(const mace_ctx* c, int32_t* count) {
  if (!c || !count) return fail(MACE_ERR_BAD_ARG, "null argument");
  *count = c->launches;
  return MACE_OK;
}

int mace_ctx_error_flag(mace_ctx* c, int32_t* flag) {
  if (!c || !flag) return fail(MACE_ERR_BAD_ARG, "null argument");
  DeviceGuard g(c->device);
  int v = 0;
  MACE_CUDA_TRY(cudaDeviceSynchronize());
  MACE_CUDA_TRY(cudaMemcpy(&v, c->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  MACE_CUDA_TRY(cudaMemset(c->d_err, 0, sizeof(int)));
  *flag = v;
  return MACE_OK;
}

}  // extern "C"
