// Halo exchange of ghost-atom rows between the ranks of a spatial domain
// decomposition, issued by the library itself on the step's stream.
//
// Each rank holds its owned atoms (local rows 0 .. n_owned-1) and ghost images
// of atoms owned by other ranks (rows n_owned .. n_local-1).  Between the two
// interaction layers the ghosts need their owners' layer-1 input features, and
// in the backward the gradients accumulated on ghost rows belong to their
// owners.  A plan (built on the host once per neighbour-list rebuild) lists,
// per peer rank, the owned rows that peer needs and, per peer, the ghost rows
// that peer fills.  Then per step:
//   features:  gather the requested owned rows into one send buffer, one NCCL
//              group of ncclSend/ncclRecv per peer, scatter the received rows
//              into the ghost rows;
//   gradients: gather the ghost rows and zero them, the reverse exchange, and
//              add the received rows onto their owned rows in a fixed order
//              (owned row by owned row, contributions in plan order), so the
//              reduction is deterministic.
// Everything runs on the caller's stream with device-resident plans, so a step
// that uses it can be captured into a CUDA graph (NCCL supports capture); the
// host-callback halo of mace_system.halo cannot.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, the library the host's
// torch build already mapped), so libmace_b200 itself has no link-time NCCL
// dependency and loads on machines without it.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <type_traits>
#include <vector>

#include "common.cuh"

namespace mace {

namespace {

struct NcclApi {
  void* so = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

int nccl_api(NcclApi** out) {
  static NcclApi api;
  static bool tried = false;
  static std::string why;
  if (!tried) {
    tried = true;
    api.so = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!api.so) {
      why = std::string("dlopen(libnccl.so.2): ") + dlerror();
    } else {
      bool ok = true;
      auto sym = [&](auto& fp, const char* name) {
        void* p = dlsym(api.so, name);
        if (!p) ok = false;
        fp = reinterpret_cast<std::remove_reference_t<decltype(fp)>>(p);
      };
      sym(api.get_unique_id, "ncclGetUniqueId");
      sym(api.comm_init_rank, "ncclCommInitRank");
      sym(api.comm_destroy, "ncclCommDestroy");
      sym(api.group_start, "ncclGroupStart");
      sym(api.group_end, "ncclGroupEnd");
      sym(api.send, "ncclSend");
      sym(api.recv, "ncclRecv");
      sym(api.error_string, "ncclGetErrorString");
      if (!ok) {
        why = "libnccl.so.2 lacks a required symbol";
        api.so = nullptr;
      }
    }
  }
  if (!api.so) return fail(MACE_ERR_NCCL, why);
  *out = &api;
  return MACE_OK;
}

#define TRY_RC(x)           \
  do {                      \
    int _rc = (x);          \
    if (_rc) return _rc;    \
  } while (0)

#define NCCL_TRY(api, expr)                                                                   \
  do {                                                                                        \
    ncclResult_t _r = (expr);                                                                 \
    if (_r != ncclSuccess) return fail(MACE_ERR_NCCL, std::string(#expr) + ": " + (api)->error_string(_r)); \
  } while (0)

// rows are float4-addressable: row_len is a multiple of 4 (C * dims, C % 32 == 0)
__global__ void k_gather_rows(const float4* __restrict__ rows, int64_t row4, const int32_t* __restrict__ idx,
                              int64_t n, float4* __restrict__ buf) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n * row4) return;
  const int64_t r = i / row4, f = i - r * row4;
  buf[i] = rows[(int64_t)idx[r] * row4 + f];
}

__global__ void k_scatter_rows(const float4* __restrict__ buf, int64_t row4, const int32_t* __restrict__ idx,
                               int64_t n, float4* __restrict__ rows) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n * row4) return;
  const int64_t r = i / row4, f = i - r * row4;
  rows[(int64_t)idx[r] * row4 + f] = buf[i];
}

__global__ void k_zero_rows(float4* __restrict__ rows, int64_t row4, const int32_t* __restrict__ idx, int64_t n) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n * row4) return;
  const int64_t r = i / row4, f = i - r * row4;
  rows[(int64_t)idx[r] * row4 + f] = make_float4(0.f, 0.f, 0.f, 0.f);
}

// rows[acc_rows[a]] += sum of buf[items[k]] for k in [ptr[a], ptr[a+1]), in that order
__global__ void k_accumulate_rows(const float4* __restrict__ buf, int64_t row4, const int32_t* __restrict__ ptr,
                                  const int32_t* __restrict__ acc_rows, const int32_t* __restrict__ items,
                                  int64_t n_acc, float4* __restrict__ rows) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_acc * row4) return;
  const int64_t a = i / row4, f = i - a * row4;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = ptr[a]; k < ptr[a + 1]; ++k) {
    const float4 v = buf[(int64_t)items[k] * row4 + f];
    s.x += v.x;
    s.y += v.y;
    s.z += v.z;
    s.w += v.w;
  }
  float4* d = rows + (int64_t)acc_rows[a] * row4 + f;
  float4 o = *d;
  o.x += s.x;
  o.y += s.y;
  o.z += s.z;
  o.w += s.w;
  *d = o;
}

unsigned blocks_for(int64_t n) { return (unsigned)((n + 255) / 256); }

}  // namespace
}  // namespace mace

struct mace_halo {
  int rank = 0, world = 1, device = 0;
  ncclComm_t comm = nullptr;
  mace::NcclApi* api = nullptr;
  int64_t n_owned = 0, n_local = 0, row_cap = 0;
  std::vector<int64_t> send_cnt, recv_cnt, send_off, recv_off;  // rows per peer
  int64_t n_send = 0, n_recv = 0, n_acc = 0;
  int32_t* d_send_rows = nullptr;  // owned rows to send, grouped by peer
  int32_t* d_recv_rows = nullptr;  // ghost rows they fill, grouped by peer
  int32_t* d_acc_ptr = nullptr;    // CSR over the owned rows that receive gradients
  int32_t* d_acc_rows = nullptr;
  int32_t* d_acc_items = nullptr;
  float* d_sbuf = nullptr;
  float* d_rbuf = nullptr;
  int version = 0;
  std::vector<void*> allocs;
  std::vector<mace_ctx*> graph_users;  // contexts whose captured step holds this halo's operations
};

namespace mace {
namespace {

void halo_free_plan(mace_halo* h) {
  for (void* p : h->allocs) cudaFree(p);
  h->allocs.clear();
  h->d_send_rows = h->d_recv_rows = h->d_acc_ptr = h->d_acc_rows = h->d_acc_items = nullptr;
  h->d_sbuf = h->d_rbuf = nullptr;
}

template <typename T>
int halo_upload(mace_halo* h, T** dst, const T* src, int64_t n) {
  void* p = nullptr;
  MACE_CUDA_TRY(cudaMalloc(&p, sizeof(T) * (size_t)(n > 0 ? n : 1)));
  h->allocs.push_back(p);
  if (n > 0) MACE_CUDA_TRY(cudaMemcpy(p, src, sizeof(T) * (size_t)n, cudaMemcpyHostToDevice));
  *dst = static_cast<T*>(p);
  return MACE_OK;
}

// one NCCL group: per peer, send cnt_s[p] rows from sbuf and receive cnt_r[p] rows into rbuf
int exchange(mace_halo* h, const std::vector<int64_t>& cnt_s, const std::vector<int64_t>& off_s,
             const std::vector<int64_t>& cnt_r, const std::vector<int64_t>& off_r, int64_t row_len,
             cudaStream_t s) {
  NcclApi* api = h->api;
  NCCL_TRY(api, api->group_start());
  for (int p = 0; p < h->world; ++p) {
    if (cnt_s[p] > 0)
      NCCL_TRY(api, api->send(h->d_sbuf + off_s[p] * row_len, (size_t)(cnt_s[p] * row_len), ncclFloat32, p, h->comm, s));
    if (cnt_r[p] > 0)
      NCCL_TRY(api, api->recv(h->d_rbuf + off_r[p] * row_len, (size_t)(cnt_r[p] * row_len), ncclFloat32, p, h->comm, s));
  }
  NCCL_TRY(api, api->group_end());
  return MACE_OK;
}

}  // namespace

int halo_features(mace_halo* h, float* rows, int64_t row_len, cudaStream_t s) {
  if (row_len > h->row_cap || row_len % 4) return fail(MACE_ERR_BAD_ARG, "halo: row longer than planned");
  const int64_t r4 = row_len / 4;
  if (h->n_send > 0)
    k_gather_rows<<<blocks_for(h->n_send * r4), 256, 0, s>>>(reinterpret_cast<const float4*>(rows), r4,
                                                              h->d_send_rows, h->n_send,
                                                              reinterpret_cast<float4*>(h->d_sbuf));
  MACE_LAUNCH_CHECK("halo_gather");
  int rc = exchange(h, h->send_cnt, h->send_off, h->recv_cnt, h->recv_off, row_len, s);
  if (rc) return rc;
  if (h->n_recv > 0)
    k_scatter_rows<<<blocks_for(h->n_recv * r4), 256, 0, s>>>(reinterpret_cast<const float4*>(h->d_rbuf), r4,
                                                               h->d_recv_rows, h->n_recv,
                                                               reinterpret_cast<float4*>(rows));
  MACE_LAUNCH_CHECK("halo_scatter");
  return MACE_OK;
}

int halo_gradients(mace_halo* h, float* rows, int64_t row_len, cudaStream_t s) {
  if (row_len > h->row_cap || row_len % 4) return fail(MACE_ERR_BAD_ARG, "halo: row longer than planned");
  const int64_t r4 = row_len / 4;
  float4* rows4 = reinterpret_cast<float4*>(rows);
  if (h->n_recv > 0) {
    k_gather_rows<<<blocks_for(h->n_recv * r4), 256, 0, s>>>(rows4, r4, h->d_recv_rows, h->n_recv,
                                                              reinterpret_cast<float4*>(h->d_sbuf));
    k_zero_rows<<<blocks_for(h->n_recv * r4), 256, 0, s>>>(rows4, r4, h->d_recv_rows, h->n_recv);
  }
  MACE_LAUNCH_CHECK("halo_gather_grad");
  // the reverse exchange: the ghost side sends (recv counts), the owner side receives (send counts)
  int rc = exchange(h, h->recv_cnt, h->recv_off, h->send_cnt, h->send_off, row_len, s);
  if (rc) return rc;
  if (h->n_acc > 0)
    k_accumulate_rows<<<blocks_for(h->n_acc * r4), 256, 0, s>>>(reinterpret_cast<const float4*>(h->d_rbuf), r4,
                                                                 h->d_acc_ptr, h->d_acc_rows, h->d_acc_items,
                                                                 h->n_acc, rows4);
  MACE_LAUNCH_CHECK("halo_accumulate");
  return MACE_OK;
}

int halo_version(const mace_halo* h) { return h ? h->version : 0; }

void halo_attach_graph(mace_halo* h, mace_ctx* c) {
  if (h && std::find(h->graph_users.begin(), h->graph_users.end(), c) == h->graph_users.end())
    h->graph_users.push_back(c);
}

void halo_detach_graph(mace_halo* h, mace_ctx* c) {
  if (h) h->graph_users.erase(std::remove(h->graph_users.begin(), h->graph_users.end(), c), h->graph_users.end());
}

}  // namespace mace

using namespace mace;

extern "C" {

int mace_halo_unique_id(void* id_out, size_t len) {
  if (!id_out || len < sizeof(ncclUniqueId)) return fail(MACE_ERR_BAD_ARG, "mace_halo_unique_id: buffer too small");
  NcclApi* api = nullptr;
  TRY_RC(nccl_api(&api));
  ncclUniqueId id;
  NCCL_TRY(api, api->get_unique_id(&id));
  std::memcpy(id_out, &id, sizeof(id));
  return MACE_OK;
}

int mace_halo_create(const void* id, size_t len, int32_t world, int32_t rank, int32_t device, mace_halo** out) {
  if (!id || !out || len < sizeof(ncclUniqueId) || world < 1 || rank < 0 || rank >= world)
    return fail(MACE_ERR_BAD_ARG, "mace_halo_create: bad arguments");
  NcclApi* api = nullptr;
  TRY_RC(nccl_api(&api));
  MACE_CUDA_TRY(cudaSetDevice(device));
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  auto* h = new mace_halo();
  h->rank = rank;
  h->world = world;
  h->device = device;
  h->api = api;
  ncclResult_t r = api->comm_init_rank(&h->comm, world, uid, rank);
  if (r != ncclSuccess) {
    delete h;
    return fail(MACE_ERR_NCCL, std::string("ncclCommInitRank: ") + api->error_string(r));
  }
  h->send_cnt.assign(world, 0);
  h->recv_cnt.assign(world, 0);
  h->send_off.assign(world, 0);
  h->recv_off.assign(world, 0);
  *out = h;
  return MACE_OK;
}

int mace_halo_plan(mace_halo* h, int64_t n_owned, int64_t n_local, int64_t row_cap, const int64_t* send_counts,
                   const int32_t* send_rows, const int64_t* recv_counts, const int32_t* recv_rows) {
  if (!h || !send_counts || !recv_counts || n_owned < 0 || n_local < n_owned || row_cap <= 0 || row_cap % 4)
    return fail(MACE_ERR_BAD_ARG, "mace_halo_plan: bad arguments");
  MACE_CUDA_TRY(cudaSetDevice(h->device));
  int64_t ns = 0, nr = 0;
  for (int p = 0; p < h->world; ++p) {
    if (send_counts[p] < 0 || recv_counts[p] < 0) return fail(MACE_ERR_BAD_ARG, "mace_halo_plan: negative count");
    h->send_off[p] = ns;
    h->recv_off[p] = nr;
    h->send_cnt[p] = send_counts[p];
    h->recv_cnt[p] = recv_counts[p];
    ns += send_counts[p];
    nr += recv_counts[p];
  }
  if ((ns > 0 && !send_rows) || (nr > 0 && !recv_rows)) return fail(MACE_ERR_BAD_ARG, "mace_halo_plan: null rows");
  for (int64_t i = 0; i < ns; ++i)
    if (send_rows[i] < 0 || send_rows[i] >= n_owned) return fail(MACE_ERR_BAD_ARG, "mace_halo_plan: send row not owned");
  for (int64_t i = 0; i < nr; ++i)
    if (recv_rows[i] < n_owned || recv_rows[i] >= n_local)
      return fail(MACE_ERR_BAD_ARG, "mace_halo_plan: receive row is not a ghost row");
  // gradient accumulation: owned rows in ascending order, each with its send positions in plan order
  std::vector<int32_t> order(ns);
  for (int64_t i = 0; i < ns; ++i) order[i] = (int32_t)i;
  std::stable_sort(order.begin(), order.end(), [&](int32_t a, int32_t b) { return send_rows[a] < send_rows[b]; });
  std::vector<int32_t> acc_ptr{0}, acc_rows;
  for (int64_t k = 0; k < ns; ++k) {
    if (k == 0 || send_rows[order[k]] != send_rows[order[k - 1]]) {
      if (k) acc_ptr.push_back((int32_t)k);
      acc_rows.push_back(send_rows[order[k]]);
    }
  }
  if (ns) acc_ptr.push_back((int32_t)ns);
  halo_free_plan(h);
  h->n_owned = n_owned;
  h->n_local = n_local;
  h->row_cap = row_cap;
  h->n_send = ns;
  h->n_recv = nr;
  h->n_acc = (int64_t)acc_rows.size();
  TRY_RC(halo_upload(h, &h->d_send_rows, send_rows, ns));
  TRY_RC(halo_upload(h, &h->d_recv_rows, recv_rows, nr));
  TRY_RC(halo_upload(h, &h->d_acc_ptr, acc_ptr.data(), (int64_t)acc_ptr.size()));
  TRY_RC(halo_upload(h, &h->d_acc_rows, acc_rows.data(), h->n_acc));
  TRY_RC(halo_upload(h, &h->d_acc_items, order.data(), ns));
  // send / receive staging (fully written before they are read)
  const int64_t nbuf = (ns > nr ? ns : nr) * row_cap;
  void* p = nullptr;
  MACE_CUDA_TRY(cudaMalloc(&p, sizeof(float) * (size_t)(nbuf > 0 ? nbuf : 4)));
  h->allocs.push_back(p);
  h->d_sbuf = static_cast<float*>(p);
  MACE_CUDA_TRY(cudaMalloc(&p, sizeof(float) * (size_t)(nbuf > 0 ? nbuf : 4)));
  h->allocs.push_back(p);
  h->d_rbuf = static_cast<float*>(p);
  ++h->version;
  return MACE_OK;
}

int mace_halo_destroy(mace_halo* h) {
  if (!h) return MACE_OK;
  cudaSetDevice(h->device);
  cudaDeviceSynchronize();
  // captured steps that hold this communicator's operations go first: NCCL's
  // destroy waits until no graph holds any
  const std::vector<mace_ctx*> users = h->graph_users;
  for (mace_ctx* c : users) ctx_drop_graph(c);
  h->graph_users.clear();
  cudaSetDevice(h->device);
  halo_free_plan(h);
  if (h->comm && h->api) h->api->comm_destroy(h->comm);
  delete h;
  return MACE_OK;
}

}  // extern "C"
