/*
 * mace_b200.h -- C ABI of the B200 MACE energy + forces + virial step.
 *
 * This is the boundary a Python (ctypes) or any other FFI caller binds to.
 * Plain pointers and sizes only; no torch or C++ types cross it.  Every entry
 * point returns a status code (MACE_OK == 0); on failure the message is kept
 * in a thread-local buffer readable with mace_last_error().
 *
 * The entry points replace the reference's compute path, which is Python on
 * MLX (mace_mlx, v0.5.0):
 *   mace_nl_build           <- calculators.py:51-62, 292-317  (_build_neighbor_list,
 *                              matscipy/ASE "ijS" list with cutoff r_max + skin)
 *   mace_forward_backward   <- calculators.py:431-483 (energy + forces through
 *                              mx.value_and_grad of model.py:440-483) and
 *                              calculators.py:489-570 (virial through the
 *                              symmetric displacement); the model body is
 *                              model.py:373-438 with blocks.py / the op modules
 *   mace_ctx_create         <- model.py:664-720 (load_model: config.json +
 *                              weights.npz) -- the host packs the converted
 *                              weights into the flat tables described below
 *
 * Conventions
 *   - All device pointers are caller-owned device memory on the context's
 *     device.  Hot calls allocate nothing; scratch lives in the context's
 *     workspace, sized by mace_ctx_reserve().
 *   - Edges are directed (sender -> receiver), sorted by receiver, with a
 *     CSR row pointer over receivers and, for every edge, the index of its
 *     reverse edge (j -> i, -S).  mace_nl_build produces exactly this.
 *     v_e = pos[receiver] - pos[sender] + shift_e @ cell  (reference utils.py:47-84).
 *   - One context per device; contexts are independent (no global state
 *     except the per-thread error string).  Calls on one context must not
 *     overlap in time on different streams.
 */
#ifndef MACE_B200_H
#define MACE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* status codes */
#define MACE_OK 0
#define MACE_ERR_BAD_ARG 1
#define MACE_ERR_CUDA 2
#define MACE_ERR_NL_OVERFLOW 3
#define MACE_ERR_TIMEOUT 4
#define MACE_ERR_NCCL 5
#define MACE_ERR_UNSUPPORTED 6
#define MACE_ERR_EDGES 7

#define MACE_ABI_VERSION 8

/* limits of the packed model description */
#define MACE_MAX_LAYERS 4
#define MACE_MAX_IN 4     /* irrep slots of a node-feature table (l <= 3)      */
#define MACE_MAX_MID 24   /* conv_tp output slots per layer                   */
#define MACE_MAX_SRC 6    /* mid slots feeding one interaction-linear output  */
#define MACE_MAX_CORR 3   /* symmetric-contraction correlation order          */

/* flags of mace_forward_backward */
#define MACE_WANT_FORCES 1
#define MACE_WANT_VIRIAL 2
/* Replay the step as a CUDA graph: captured on the first call (and whenever
 * any pointer, size or flag of the call changes), then launched on `stream`.
 * Buffers must keep their addresses between calls; mace_ctx_reserve drops
 * the captured graph.  Ignored while profiling is enabled. */
#define MACE_USE_GRAPH 4

typedef struct mace_ctx mace_ctx;

/* Offsets below index the float table `floats` (f_*) or the int table `ints`
 * (i_*) of mace_model_desc.  Node-feature tables are stored channel-last per
 * irrep slot: row n, slot s, component m, channel u at
 * n*dim + off[s] + m*C + u.  Weights have their path weights folded in. */

typedef struct {
  int32_t n;                      /* number of slots                    */
  int32_t l[MACE_MAX_IN];         /* degree of each slot                */
  int32_t off[MACE_MAX_IN];       /* offset of each slot within a row   */
  int32_t dim;                    /* row length = C * sum(2l+1)         */
} mace_slots;

typedef struct {
  int32_t l1, l2, l3;             /* degrees of x1 (node), Y (edge), out */
  int32_t src;                    /* input slot of x1                   */
  int32_t off;                    /* offset of this slot in the mid row */
  int32_t m_off;                  /* offset of its (2l1+1)(2l3+1) block in a per-edge M row */
  int64_t f_cg;                   /* path-weighted 3j, (2l1+1)(2l2+1)(2l3+1) */
} mace_conv_slot;

typedef struct {
  int32_t n_src;                  /* mid slots with this degree         */
  int32_t src[MACE_MAX_SRC];      /* their indices                      */
  int64_t f_w;                    /* (n_src*C, C) row-major, concat-K   */
  int64_t f_wt;                   /* (C, n_src*C) transpose             */
} mace_lin_group;

/* Symmetric contraction of one output irrep, as a polynomial in the coupling
 * features f[i] (i = l^2 + m): out[M][c] = sum_e G[z][e][c] * f[a_e] (* f[b_e] (* f[c_e]))
 * over entries e with sorted indices a <= b <= c; G already contains the
 * species weights contracted with the index-symmetrised U tensors. */
typedef struct {
  int32_t L;                      /* output degree                      */
  int32_t corr;                   /* correlation order                  */
  int32_t n_ent;                  /* number of entries                  */
  int64_t i_ent;                  /* ints: (2L+2) segment starts by M, then n_ent packed
                                     M | a<<4 | b<<8 | c<<12 | nu<<16 */
  int64_t f_G;                    /* floats: (num_elements, n_ent, C)    */
} mace_sc_out;

typedef struct {
  int32_t C;                      /* channels (multiplicity)            */
  int32_t residual;               /* 1: skip before message; 0: skip on message */
  mace_slots in;                  /* layer input irreps                 */
  mace_slots hid;                 /* product output irreps              */
  mace_slots mid;                 /* conv_tp output row: only `dim` is used (slots are in conv[]) */
  mace_slots inter;               /* interaction irreps 0..lmax         */
  /* skip_tp: species-indexed (num_elements, C, C) blocks per pair in->out */
  int32_t n_skip;
  int32_t skip_in[MACE_MAX_IN], skip_out[MACE_MAX_IN];
  int64_t f_skip[MACE_MAX_IN], f_skip_t[MACE_MAX_IN];
  /* linear_up: one (C, C) block per input slot (1-to-1) */
  int64_t f_up[MACE_MAX_IN], f_up_t[MACE_MAX_IN];
  /* radial MLP */
  int32_t n_mlp;                  /* number of Linear layers            */
  int32_t mlp_w[8];               /* widths: in, hidden..., out         */
  int64_t f_mlp[7], f_mlp_t[7];   /* (in, out) and (out, in) per layer   */
  /* MLP layers as tensor-core operand images (hidden width 64, <= 16 radial
   * features; else -1), tf32 hi then lo, each 128B-swizzled K-major:
   * last layer forward: per 32-output chunk the (32 x 64) slice of (out, in);
   * last layer backward: per 32-output chunk the (64 x 32) slice of (in, out);
   * hidden layers 1..: (out, in) for the forward, (in, out) for the backward. */
  int64_t f_mlp_tc, f_mlp_tc_bwd, f_mlp_tc_trunk, f_mlp_tc_trunk_bwd;
  /* conv_tp */
  int32_t n_mid;
  int32_t m_tot;                  /* length of a per-edge M row          */
  int32_t wnumel;                 /* per-edge weights = n_mid * C        */
  mace_conv_slot conv[MACE_MAX_MID];
  /* interaction linear (mid -> inter), one group per output degree */
  mace_lin_group lin[MACE_MAX_IN];
  /* symmetric contraction: one entry per hidden slot */
  mace_sc_out sc[MACE_MAX_IN];
  /* symmetric-contraction backward as one polynomial per coupling index k:
   *   df[k][c] = sum_e G'[z][e][c] * g[r_e][c] (* f[b_e] (* f[c_e]))
   * where g is the product-output gradient, r = (slot offset / C) + M its row,
   * and G' = (multiplicity of k in the forward entry) x G. */
  int32_t sc_n_bwd;               /* number of backward entries         */
  int64_t i_sc_bwd;               /* ints: (ncoup+1) segment starts by k, then packed
                                     b | c<<4 | nu'<<8 | r<<10 (nu' = degree - 1) */
  int64_t f_sc_bwd;               /* floats: (num_elements, sc_n_bwd, C) */
  /* 1, 2, 3: the product outputs are (0e), (0e, 1o), (0e, 1o, 2e) with the
   * standard entry lists (16 coupling features, correlation 3), served by the
   * generated straight-line kernels; 0: table-driven kernels */
  int32_t sc_gen;
  /* product linear: one (C, C) block per hidden slot */
  int64_t f_prod[MACE_MAX_IN], f_prod_t[MACE_MAX_IN];
  /* readout */
  int32_t readout_nonlinear;
  int32_t readout_hidden;         /* 16 */
  int64_t f_ro1;                  /* linear: (C); nonlinear: (C, hidden) */
  int64_t f_ro2;                  /* nonlinear: (hidden)                 */
  /* density normalisation (reference blocks.py:282-490): the message is
   * divided by (sum over the receiver's edges of tanh((w_d . b_e)^2) + 1)
   * instead of avg_num_neighbors; f_density = w_d (num_bessel), else -1 */
  int32_t density;
  int64_t f_density;
} mace_layer_desc;

typedef struct {
  int32_t abi_version;            /* MACE_ABI_VERSION                    */
  int32_t num_layers;
  int32_t num_elements;
  int32_t num_bessel;
  int32_t max_ell;                /* <= 3                                */
  int32_t poly_p;
  int32_t scale_shift;            /* 1: ScaleShiftMACE energy assembly   */
  int32_t C;
  float r_max;
  float inv_avg_num_neighbors;
  float scale, shift;
  int64_t f_e0;                   /* (num_elements) atomic energies      */
  int64_t f_emb;                  /* (num_elements, C) embedding, 1/sqrt(E) folded */
  int64_t f_bessel;               /* (num_bessel) frequencies            */
  int64_t f_sh;                   /* SH recursion tensors T_2, T_3       */
  mace_layer_desc layers[MACE_MAX_LAYERS];
  /* Agnesi distance transform of the length fed to the Bessel basis
   * (reference radial.py:202-262): r_t = 1 / (1 + a x^q / (1 + x^(q-p))),
   * x = max(r / r0, 1e-12), r0 = (R[z_s] + R[z_r]) / 2 with R of f_radius_agnesi */
  int32_t agnesi;
  float agnesi_q, agnesi_p, agnesi_a;
  int64_t f_radius_agnesi;        /* (num_elements) covalent radius per element index */
  /* ZBL pair repulsion (reference radial.py:127-199), added to the receiver's
   * interaction energy: 0.5 * 14.3996 Z_s Z_r / r * phi(r / a) * envelope_p(r / (R_s + R_r)),
   * a = a_prefactor * 0.529 / (Z_s^a_exp + Z_r^a_exp) */
  int32_t zbl;
  int32_t zbl_p;
  float zbl_a_exp, zbl_a_prefactor;
  int64_t f_radius_zbl;           /* (num_elements) covalent radius per element index */
  int64_t f_znum;                 /* (num_elements) atomic number per element index (float) */
  /* 1: apply_cutoff=False models (reference radial.py:294-321, blocks.py:163-164):
   * the polynomial envelope multiplies each edge's radial-MLP output instead of
   * its Bessel features; not combined with density-normalised layers */
  int32_t envelope_on_weights;
  int32_t reserved0;
  const float* floats; int64_t n_floats;    /* host pointers, copied at create */
  const int32_t* ints; int64_t n_ints;
} mace_model_desc;

/*
 * Halo exchange between interaction layers (spatial domain decomposition).
 * Called on the host, in stream order, with the device rows of all nodes
 * (row_len floats per node, node-major) and the stream of the step:
 *   phase MACE_HALO_FEATURES:  after layer `layer` produced its node features;
 *     the callee overwrites the ghost rows with their owners' rows.
 *   phase MACE_HALO_GRADIENTS: after the backward produced the gradient of the
 *     energy w.r.t. the input features of layer `layer` + 1; the callee adds
 *     the ghost rows into their owners' rows (on the owning ranks) and zeroes
 *     the ghost rows.
 * Return 0, or non-zero to abort the step (reported as MACE_ERR_NCCL).
 * Not used under MACE_USE_GRAPH.
 */
/* In-library halo exchange over NCCL (see mace_halo_create); opaque. */
typedef struct mace_halo mace_halo;

#define MACE_HALO_FEATURES 0
#define MACE_HALO_GRADIENTS 1
typedef int (*mace_halo_fn)(void* user, int32_t phase, int32_t layer, float* rows, int64_t row_len, void* stream);

/* Device pointers describing one (batch of) structure(s). */
typedef struct {
  int64_t n_nodes;
  int64_t n_edges;
  int32_t num_graphs;
  const float* pos;               /* (n_nodes, 3)                        */
  const float* cell;              /* (9) row-major lattice vectors, may be NULL if no shifts */
  const int32_t* species;         /* (n_nodes) model element index       */
  const int32_t* graph_ptr;       /* (num_graphs + 1) node ranges per graph */
  const int32_t* sender;          /* (n_edges)                           */
  const int32_t* receiver;        /* (n_edges) non-decreasing            */
  const int32_t* shifts;          /* (n_edges, 3) integer lattice shifts */
  const int32_t* row_ptr;         /* (n_nodes + 1) CSR over receivers    */
  const int32_t* rev;             /* (n_edges) index of the reverse edge */
  /* (n_nodes) weight of each node's energy in the graph energies and hence in
   * every gradient, or NULL for all 1.  Spatial domain decomposition gives
   * owned atoms 1 and ghost atoms 0. */
  const float* energy_weight;
  /* The per-edge radial work runs in n_chunks consecutive receiver ranges
   * (0 or 1: one range), so the per-edge weight buffers only hold one chunk
   * (mace_ctx_reserve_chunked); with several chunks the backward recomputes
   * the radial MLP of each chunk.  Host arrays of n_chunks + 1 entries:
   * receiver boundaries (0 .. n_nodes) and row_ptr at those receivers. */
  int32_t n_chunks;
  const int64_t* chunk_nodes;
  const int64_t* chunk_edges;
  /* halo exchange between layers, or NULL (see mace_halo_fn) */
  mace_halo_fn halo;
  void* halo_user;
  /* Receivers [0, n_active) are evaluated; 0 means all.  Nodes at and beyond
   * n_active (ghost atoms of a domain decomposition) take part only as
   * senders: no conv, product, readout or energy work is done for them, their
   * energy weights must be 0, and the edges they receive (the suffix of the
   * receiver-sorted list after row_ptr[n_active], which the caller passes as
   * e_active) get no radial work. */
  int64_t n_active;
  int64_t e_active;
  /* In-library halo exchange between layers (NCCL send/recv on the step's
   * stream, capturable into the step's CUDA graph), or NULL.  Used instead of
   * `halo` when set. */
  mace_halo* halo_exchange;
} mace_system;

/* Device pointers receiving the results (NULL = not wanted). */
typedef struct {
  double* energy;                 /* (num_graphs)                        */
  float* node_energy;             /* (n_nodes)                           */
  float* forces;                  /* (n_nodes, 3) = -dE/dpos              */
  double* virial;                 /* (9) sum_e v_e (x) dE/dv_e (un-symmetrised) */
} mace_outputs;

/*
 * Halo exchange of a spatial domain decomposition inside the library (no
 * reference counterpart: the reference runs on one device).  One object per
 * rank; all ranks of the decomposition create theirs together:
 *   mace_halo_unique_id   on one rank (128 bytes), shared with the others by the caller
 *   mace_halo_create      on every rank (collective: NCCL communicator init)
 *   mace_halo_plan        on every rank after each neighbour-list rebuild
 *                         (allocates; not a hot call); per peer p in rank order:
 *                         send_rows: the owned local rows p needs (send_counts[p]),
 *                         recv_rows: the local ghost rows p fills (recv_counts[p]),
 *                         in the order p sends them; row_cap: the longest row
 *                         exchanged (floats, a multiple of 4)
 *   mace_system.halo_exchange = the object, for every step
 *   mace_halo_destroy     on every rank; first releases the captured step
 *                         graphs of the contexts that hold this halo's NCCL
 *                         operations (NCCL's destroy waits until none does)
 * Per step, after each layer but the last, the ghost rows of the node features
 * are overwritten with their owners' rows; in the backward the ghost rows of
 * the feature gradients are added onto their owners' rows (in a fixed order)
 * and zeroed.  NCCL (libnccl.so.2) is loaded on first use.
 */
int mace_halo_unique_id(void* id_out, size_t len);
int mace_halo_create(const void* id, size_t len, int32_t world, int32_t rank, int32_t device, mace_halo** out);
int mace_halo_plan(mace_halo* h, int64_t n_owned, int64_t n_local, int64_t row_cap, const int64_t* send_counts,
                   const int32_t* send_rows, const int64_t* recv_counts, const int32_t* recv_rows);
int mace_halo_destroy(mace_halo* h);

/* Message of the last failed call on this thread (always NUL-terminated). */
int mace_last_error(char* buf, size_t len);

/* Copy the packed model to `device` and create a context. */
int mace_ctx_create(const mace_model_desc* desc, int device, mace_ctx** out);
int mace_ctx_destroy(mace_ctx* ctx);

/* Size the workspace for systems up to max_nodes / max_edges (allocates; not a hot call). */
int mace_ctx_reserve(mace_ctx* ctx, int64_t max_nodes, int64_t max_edges);

/* As mace_ctx_reserve, with the per-edge radial-weight buffers sized for
 * edge chunks of at most max_chunk_edges edges (see mace_system.n_chunks). */
int mace_ctx_reserve_chunked(mace_ctx* ctx, int64_t max_nodes, int64_t max_edges, int64_t max_chunk_edges);

/* Bytes of device workspace the context currently holds. */
int mace_ctx_workspace_bytes(const mace_ctx* ctx, int64_t* bytes);

/*
 * Neighbour list on the GPU: every (i, j, S) with |x_j - x_i + S @ cell| < r_cut,
 * except i == j with S == 0, restricted to pairs in the same graph; S is zero
 * along non-periodic axes.  The distance test runs in float64.
 *   pos        (n, 3) float64 device, cell (9) float64 device (ignored if no pbc)
 *   pbc        three host ints
 *   graph_ptr  (num_graphs + 1) int32 device
 * Outputs (device, capacity entries): sender, receiver, shifts (capacity, 3),
 * row_ptr (n + 1), rev.  Edges are sorted by (receiver, sender, S).
 * *n_edges (host) receives the edge count.  Returns MACE_ERR_NL_OVERFLOW, with
 * *n_edges set to the required capacity, when capacity is too small.
 * Synchronises `stream` (the count is returned to the host).
 */
int mace_nl_build(mace_ctx* ctx, const double* pos, const double* cell, const int32_t* pbc,
                  const int32_t* graph_ptr, int32_t num_graphs, int64_t n, double r_cut,
                  int32_t* sender, int32_t* receiver, int32_t* shifts, int32_t* row_ptr,
                  int32_t* rev, int64_t capacity, int64_t* n_edges, void* stream);

/*
 * Neighbour list for callers that cannot allocate device memory (no reference
 * counterpart: the reference always builds its list on the host).  Same
 * inputs, outputs, ordering and status codes as mace_nl_build, but no context:
 * its scratch is a static __device__ array of MACE_NOALLOC_SCRATCH_BYTES that
 * every GPU loading the library holds until exit, so it works for hosts that
 * own all GPU memory or cannot afford cudaMalloc's implicit synchronisation.
 * Calls nothing that allocates.  Limits: at most MACE_NOALLOC_MAX_ATOMS atoms
 * in total and MACE_NOALLOC_MAX_GRAPH_ATOMS per graph (larger systems fail
 * with MACE_ERR_BAD_ARG).  Cost: always the all-pairs build, O(n_g^2 x periodic
 * images) per graph of n_g atoms (mace_nl_build switches to cell lists for
 * large single structures).  With CUDA's default lazy module loading the first
 * call on a device loads the array (4 MiB): make it before a memory pool takes
 * all free memory (or set CUDA_MODULE_LOADING=EAGER), and before any stream
 * capture.  The array's device address is cached per device and CUDA context.
 * All calls share the array: calls that overlap on the GPU race.
 * Uses the caller's current device.
 */
#define MACE_NOALLOC_SCRATCH_BYTES (4u << 20)
#define MACE_NOALLOC_MAX_ATOMS 131072
#define MACE_NOALLOC_MAX_GRAPH_ATOMS 16384
int mace_nl_build_noalloc(const double* pos, const double* cell, const int32_t* pbc,
                          const int32_t* graph_ptr, int32_t num_graphs, int64_t n, double r_cut,
                          int32_t* sender, int32_t* receiver, int32_t* shifts, int32_t* row_ptr,
                          int32_t* rev, int64_t capacity, int64_t* n_edges, void* stream);

/*
 * One energy (+ forces, + virial) evaluation on `stream` (a cudaStream_t).
 * Asynchronous: results are valid once the stream reaches this point.  An
 * inconsistent reverse-edge index is recorded in the context's error flag
 * (see mace_ctx_error_flag); the forces of the affected atoms are then wrong.
 */
int mace_forward_backward(mace_ctx* ctx, const mace_system* sys, const mace_outputs* out,
                          int32_t flags, void* stream);

/*
 * Debug/parity access to an internal per-stage buffer after the last call:
 * id = layer * 16 + stage (see mace_mlx_b200/native.py for the stage list).
 * Returns the device pointer and length in floats.  The radial weights
 * (stage "w") are in 128-edge tiles: tile e / 128 holds ceil(W / 32) chunks
 * of 128 rows x 32 floats; column c of edge e sits in chunk c / 32 at row
 * e % 128, 16-byte group ((c % 32) / 4) XOR (e % 8), position c % 4.
 */
int mace_debug_buffer(mace_ctx* ctx, int32_t id, const float** ptr, int64_t* len);

/*
 * Diagnostic (no reference counterpart): FP32 fused multiply-add issue-rate
 * probe used to measure the CUDA-core peak the benchmark's roofline compares
 * CUDA-core kernels with.  Launches `blocks` CTAs of 256 threads, each thread
 * running 8 independent FMA chains of 16 x `iters` steps (FLOPs = blocks x 256
 * x 8 x 16 x iters x 2) and writing one float per thread to `out`
 * (blocks x 256 floats, device memory).  Asynchronous on `stream`.
 */
int mace_fma_probe(float* out, int32_t blocks, int32_t iters, void* stream);

/* Number of kernel launches the last mace_forward_backward issued. */
int mace_last_launch_count(const mace_ctx* ctx, int32_t* count);

/*
 * Opt-in timing of every launch with CUDA events recorded on the launching
 * stream (for benchmarks; adds an event pair per kernel).  Enabling resets the
 * totals.  mace_profile_read synchronises, then returns per (kernel, layer):
 * name (32 bytes each in `names`), layer (-1 = not per layer), launch count and
 * total milliseconds since the previous read.
 */
int mace_profile_enable(mace_ctx* ctx, int32_t enable);
int mace_profile_read(mace_ctx* ctx, int32_t max_entries, char* names, int32_t* layers,
                      int32_t* counts, double* total_ms, int32_t* n_entries);
/* The last profiled step's launches in issue order: name, layer, stream (0 =
 * the caller's, 1 = the runtime's second stream), start and end in
 * milliseconds from the step's first launch. */
int mace_profile_timeline(mace_ctx* ctx, int32_t max_entries, char* names, int32_t* layers,
                          int32_t* streams, float* start_ms, float* end_ms, int32_t* n_entries);

/* Synchronise the device, return and clear the context's device error flag
 * (1 = an edge's reverse index did not point back to it). */
int mace_ctx_error_flag(mace_ctx* ctx, int32_t* flag);

#ifdef __cplusplus
}
#endif
#endif /* MACE_B200_H */
