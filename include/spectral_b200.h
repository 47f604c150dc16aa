/*
 * spectral_b200.h — C ABI of libspectral_b200.so (B200 / sm_100a).
 *
 * The drop-in boundary for SpectralAI's MoE inference hot path:
 *   - the BVH expert router (eval forward of BVHRouter, python/bvh_router.py:269-329),
 *   - the ternary {-1,0,+1} SwiGLU expert (ternary_gated_mlp,
 *     cuda/v5/ternary_torch_ext.cu:123-191, 284-339) and its grouped MoE form.
 *
 * Conventions
 *   - Plain pointers and sizes only.  Device pointers are CUDA device addresses
 *     on the handle's device; `stream` is a cudaStream_t passed as void*.
 *   - Every entry point returns an int status: SB_OK (0) or a negative SB_ERR_*.
 *     The message of the last failure on the calling thread is available from
 *     sb_last_error().  Nothing here calls exit/abort or traps on the device.
 *   - Forward calls are asynchronous on `stream` (like the reference's
 *     bvh_router_ext.route, cuda/v5/bvh_torch_ext.cu:310-357).
 *   - The caller owns all input/output buffers and the workspace; a handle owns
 *     only its device-resident weights.  Handles are independent (no process-
 *     global tree, unlike the reference's __constant__ tree,
 *     cuda/v5/bvh_torch_ext.cu:51-55), so one process may hold many routers.
 *   - Device kernels bound every wait; a wait that runs out sets a status word
 *     that the next call returns as SB_ERR_DEVICE_TIMEOUT.
 */
#ifndef SPECTRAL_B200_H
#define SPECTRAL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SB_ABI_VERSION 1

enum sb_status {
  SB_OK = 0,
  SB_ERR_INVALID = -1,        /* bad argument (null, shape, dtype, mode)          */
  SB_ERR_CUDA = -2,           /* CUDA runtime / driver error                       */
  SB_ERR_UNSUPPORTED = -3,    /* valid but not supported by this build           */
  SB_ERR_DEVICE_TIMEOUT = -4, /* a bounded device-side wait expired              */
  SB_ERR_NOMEM = -5,          /* device allocation failed                        */
  SB_ERR_WORKSPACE = -6       /* workspace smaller than *_workspace_bytes()       */
};

enum sb_dtype { SB_F32 = 0, SB_BF16 = 1, SB_F16 = 2 };

/* Level selection rule.  HARD = the reference eval branch (argmax + one_hot,
 * bvh_router.py:190-193).  SOFT = the training branch with the Gumbel noise
 * removed, softmax(logits / clamp(T, 0.01)) (bvh_router.py:200-202). */
enum sb_select { SB_SELECT_HARD = 0, SB_SELECT_SOFT = 1 };

/* Arithmetic of the encoder GEMMs.  FAST = bf16 tcgen05 tensor cores with fp32
 * accumulation (input must be bf16); EXACT = fp32 FFMA (input fp32 or bf16),
 * matching the reference's fp32 PyTorch math to rounding. */
enum sb_precision { SB_PREC_FAST = 0, SB_PREC_EXACT = 1 };

/* Version of this ABI (SB_ABI_VERSION). */
int sb_abi_version(void);

/* Copies the calling thread's last error message (NUL-terminated) into buf.
 * Returns the full message length. */
int sb_last_error(char* buf, size_t len);

/* Reads and clears the device status word of `device` (synchronous).  Returns
 * SB_OK or SB_ERR_DEVICE_TIMEOUT if a kernel gave up a bounded wait. */
int sb_device_status(int device);

/* Per-kernel timing with CUDA events recorded on each launch's stream (the
 * reference times host-side with perf_counter + synchronize,
 * python/benchmark_cuda_pipeline.py:110-146).  Enabling clears the counters. */
int sb_profile_enable(int on);
/* Number of distinct kernels timed so far (waits for the recorded events). */
int sb_profile_count(void);
/* Name, launch count and summed milliseconds of timed kernel i. */
int sb_profile_entry(int i, char* name, size_t len, int64_t* launches, double* total_ms);

/* ------------------------------------------------------------------------ */
/* BVH router                                                                */
/* ------------------------------------------------------------------------ */

#define SB_MAX_LEVELS 8

typedef struct sb_router sb_router;

/* Router shape.  Replaces RouterConfig (python/bvh_router.py:28-65), with the
 * three hard-coded levels generalised to n_levels (1..8). */
typedef struct {
  int32_t hidden;                    /* embed_dim H                         */
  int32_t spectral;                  /* spectral_dim S                      */
  int32_t n_levels;                  /* L (reference: 3)                    */
  int32_t branching[SB_MAX_LEVELS];  /* children per node at each level     */
} sb_router_desc;

/* Host fp32 parameters in the reference state_dict layout
 * (python/bvh_router.py:227-255).  Level l (0-based) has N_l = prod(branching[0..l]) nodes.
 * Null biases read as zero.  portals[l] is required for l < n_levels-1. */
typedef struct {
  const float* to3d_w;                      /* to_3d.weight            [3,H]     */
  const float* to3d_b;                      /* to_3d.bias              [3]       */
  const float* enc1_w;                      /* spectral.net.0.weight   [H,H]     */
  const float* enc1_b;                      /* spectral.net.0.bias     [H]       */
  const float* enc2_w;                      /* spectral.net.2.weight   [S,H]     */
  const float* enc2_b;                      /* spectral.net.2.bias     [S]       */
  const float* centers[SB_MAX_LEVELS];      /* level{l+1}.centers      [N_l,3]   */
  const float* refract_w[SB_MAX_LEVELS];    /* refract{l+1}.W_dispersion.weight [N_l,S] */
  const float* refract_b[SB_MAX_LEVELS];    /* refract{l+1}.W_dispersion.bias   [N_l]   */
  const float* portals[SB_MAX_LEVELS];      /* portal{l+1}.transform   [N_l,3,4] */
  float temperature;                        /* buffer `temperature`              */
} sb_router_weights;

/* Output buffers of one forward (device pointers; any may be NULL to skip).
 * Mirrors RoutingResult (bvh_router.py:72-77) plus the MoE top-k pair. */
typedef struct {
  int32_t* topk_ids;      /* [B,k]   top-k experts, larger prob first, ties -> lower id */
  float* topk_weights;    /* [B,k]   softmax over the k selected probabilities          */
  int64_t* expert_id;     /* [B]     argmax of the last level                           */
  float* expert_probs;    /* [B,N_L] last-level probabilities                           */
  int64_t* route_path;    /* [B,L]   level-global chosen node per level                 */
  float* confidence;      /* [B]     max of the last level                              */
} sb_router_outputs;

/* Creates a router on `device`.  Replaces BVHRouter.__init__ (bvh_router.py:227-255)
 * and the reference C-ABI's bvh_alloc_buffers (cuda/v5/bvh_router_kernel.cu:378-717). */
int sb_router_create(const sb_router_desc* desc, int device, sb_router** out);

/* Copies host fp32 parameters into handle-owned device memory (synchronous).
 * Replaces bvh_router_ext.upload_tree (cuda/v5/bvh_torch_ext.cu:270-303). */
int sb_router_upload(sb_router* h, const sb_router_weights* w);

/* Bytes of caller-provided device workspace that sb_router_forward needs. */
size_t sb_router_workspace_bytes(const sb_router* h, int64_t batch, int precision);

/* Router forward over x [B,H] (device, row-major, dtype SB_F32 or SB_BF16).
 * Replaces BVHRouter.forward in eval mode (bvh_router.py:269-329) and the
 * reference kernel launch bvh_router_ext.route (cuda/v5/bvh_torch_ext.cu:310-357).
 * No batch cap (the reference caps B at 1024). */
int sb_router_forward(sb_router* h, const void* x, int x_dtype, int64_t batch,
                      int precision, int select, int top_k,
                      const sb_router_outputs* out,
                      void* workspace, size_t workspace_bytes, void* stream);

int sb_router_destroy(sb_router* h);

/* Size of the fixed device array behind sb_router_forward_noalloc (32 MiB per GPU). */
#define SB_ROUTER_NOALLOC_SCRATCH_BYTES (32u << 20)

/* Router forward that allocates nothing; no counterpart in the reference.
 * Same arguments and outputs as sb_router_forward minus the workspace: its
 * scratch is a fixed 32 MiB device array inside the library, for callers that
 * cannot allocate device memory when they route (a serving process whose HBM
 * is all reserved by its own pool, or a language runtime binding this ABI with
 * no device allocator).  Limits and sharing:
 *   - batch is limited to sb_router_workspace_bytes(h, batch, precision) below
 *     the array size minus up to 768 bytes of alignment (about 6500 tokens at
 *     hidden 2048 in SB_PREC_FAST); larger batches fail with SB_ERR_INVALID;
 *   - every GPU that loads the library holds the array until the process exits;
 *   - the first call on a device looks up the array's device address (once per
 *     device, with that device current); make that first call before any
 *     stream capture;
 *   - all calls share the one array per device and it keeps the last call's
 *     contents (nothing needs clearing: each call writes every scratch element
 *     it reads); calls that overlap on the GPU, e.g. on two streams, race. */
int sb_router_forward_noalloc(sb_router* h, const void* x, int x_dtype, int64_t batch,
                              int precision, int select, int top_k,
                              const sb_router_outputs* out, void* stream);

/* ------------------------------------------------------------------------ */
/* Ternary experts                                                           */
/* ------------------------------------------------------------------------ */

/* Host packer in the reference layout: int8 w[K,N] in {-1,0,+1} -> int32
 * packed[ceil(K/16), N], 2-bit codes 00=0, 01=+1, 10=-1, bit pair i of word
 * [p,c] = row p*16+i.  Replaces pack_ternary_impl (ternary_torch_ext.cu:197-231). */
int sb_ternary_pack_ref(const int8_t* w, int64_t K, int64_t N, int32_t* packed);

/* Bytes of one matrix in the device layout used by the B200 kernels: row-major
 * [N, ceil(K/64)*4] uint32 words, one word per 16 consecutive K of one output
 * row n.  Inside a word, element 2j+e (j=0..7, e=0,1) is the biased code
 * value+1 in {0,1,2} at bits 16e+p..16e+p+1 with p = 0,2,4,8,10,12,6,14 for
 * j = 0..7 (padding: code 1), so that two elements expand to two 16-bit floats
 * with an and-or and one packed subtraction (plus a shift for the pairs that
 * lie beyond the format's mantissa). */
size_t sb_ternary_matrix_bytes(int64_t K, int64_t N);

/* Converts a reference-layout packed matrix (device int32 [ceil(K/16), N]) into
 * the device layout above (device buffer of sb_ternary_matrix_bytes(K,N)). */
int sb_ternary_repack(const int32_t* packed_ref, int64_t K, int64_t N,
                      uint32_t* dst, void* stream);

/* Fused ternary gated MLP for one expert: y[M,H] = s_d * (T_d (silu(s_g*(T_g x)) * (s_u*(T_u x)))).
 * x: device [M,H] (SB_F32 or SB_BF16); weights in the device layout
 * (gate/up: K=H, N=I; down: K=I, N=H); scales fp32 [I],[I],[H]; y: fp32 [M,H].
 * Replaces ternary_gated_mlp (ternary_torch_ext.cu:284-339). */
int sb_ternary_gated_mlp(const void* x, int x_dtype, int64_t M, int64_t H, int64_t I,
                         const uint32_t* gate, const uint32_t* up, const uint32_t* down,
                         const float* gate_scale, const float* up_scale, const float* down_scale,
                         float* y, void* workspace, size_t workspace_bytes, void* stream);

size_t sb_ternary_gated_mlp_workspace_bytes(int64_t M, int64_t H, int64_t I);

/* y[M,N] = scale * (x @ T) + bias with x [M,K] (SB_F32/SB_BF16) and T in the device layout.
 * Replaces ternary_linear (ternary_torch_ext.cu:237-278). */
int sb_ternary_linear(const void* x, int x_dtype, int64_t M, int64_t K, int64_t N,
                      const uint32_t* w, const float* scale, const float* bias,
                      float* y, void* workspace, size_t workspace_bytes, void* stream);

size_t sb_ternary_linear_workspace_bytes(int64_t M, int64_t K, int64_t N);

/* Grouped MoE SwiGLU over E experts with top-k routing:
 *   out[t] = sum_j weights[t,j] * expert_{ids[t,j]}(x[t])
 * The k terms of a token are added along a binary tree over the expert ids
 * (two partial sums meet where their experts' indices first differ, deepest
 * bit first), the order the expert-parallel layer below reproduces across GPUs.
 * Replaces the reference's per-(slot, expert) Python loop OLMoELayer.forward_topk
 * (python/olmoe_extract.py:126-157) over CUDATernaryExpertModule experts.
 * x: device [B,H] (SB_F32/SB_BF16); ids int32 [B,k] (each in [0,E)); weights fp32 [B,k];
 * gate/up/down: device arrays of E matrices in the device layout, contiguous per kind
 * (expert e at offset e*sb_ternary_matrix_bytes); scales fp32 [E,I],[E,I],[E,H];
 * out: device [B,H] of out_dtype (SB_F32 or SB_BF16). */
int sb_ternary_moe_swiglu(const void* x, int x_dtype, int64_t B, int64_t H, int64_t I,
                          int32_t n_experts, int32_t top_k,
                          const int32_t* ids, const float* weights,
                          const uint32_t* gate, const uint32_t* up, const uint32_t* down,
                          const float* gate_scale, const float* up_scale, const float* down_scale,
                          void* out, int out_dtype,
                          void* workspace, size_t workspace_bytes, void* stream);

size_t sb_ternary_moe_workspace_bytes(int64_t B, int64_t H, int64_t I,
                                      int32_t n_experts, int32_t top_k);

/* ------------------------------------------------------------------------ */
/* Expert-parallel MoE layer over the GPUs of one node                       */
/* ------------------------------------------------------------------------ */
/* The grouped ternary SwiGLU with the experts spread over W ranks (one
 * process per GPU, W <= 8): rank r holds experts [r*E/W, (r+1)*E/W).  The
 * layer's own kernels move each token row once to every rank that holds one of
 * its experts, and the expert outputs back, through peer memory (NVLink /
 * NVSwitch; CUDA IPC mappings), with no host synchronisation on the data path.
 * The output equals sb_ternary_moe_swiglu on one GPU bit for bit when E/W is
 * a power of two (same kernels per row, same summation tree).
 * Replaces the reference's per-slot dispatch loop (python/olmoe_extract.py:
 * 146-155) and its scatter / weighted-combine kernels (cuda/async_pipeline.cu:
 * 79-133) when the experts do not all live on one GPU; the reference has no
 * multi-GPU code.
 *
 * Set-up (collective over the W ranks):
 *   sb_ep_create        on each rank, with its GPU current; allocates the
 *                       peer-visible receive buffers (W * max_tokens rows each
 *                       way) and a control block;
 *   sb_ep_connect_nccl  exchanges the buffers' IPC handles over an NCCL
 *                       communicator of the same W ranks (an ncclComm_t passed
 *                       as void*, like the streams), or
 *   sb_ep_export / sb_ep_connect  the same exchange done by the caller: each
 *                       rank's SB_EP_HANDLE_BYTES bytes, gathered in rank order.
 * Forward (collective: every rank calls it, equally often, any batch <=
 * max_tokens including 0): x bf16 [B,H]; ids int32 [B,k] in [0,E); weights
 * fp32 [B,k]; gate/up/down and scales: this rank's E/W experts in the layout
 * of sb_ternary_moe_swiglu; out [B,H] SB_F32 or SB_BF16; workspace of
 * sb_ep_workspace_bytes(h) bytes (1024-byte aligned), owned by the caller.
 * Every wait for a peer is bounded by timeout_ms; one that runs out is
 * reported by sb_ep_status (SB_ERR_DEVICE_TIMEOUT), after which the handle
 * must be destroyed and the layer set up again.
 * Tear-down: all ranks call sb_ep_destroy after a barrier (a rank's buffers
 * stay mapped by its peers until they destroy theirs). */
typedef struct sb_ep sb_ep;

typedef struct {
  int32_t world;        /* ranks W, 1..8 */
  int32_t rank;         /* this process's rank */
  int32_t n_experts;    /* E, a multiple of W, at most 255 per rank */
  int32_t top_k;        /* k, 1..16 */
  int64_t max_tokens;   /* tokens per rank per forward, at most */
  int64_t hidden;       /* H, a multiple of 8 */
  int64_t intermediate; /* I */
  int32_t timeout_ms;   /* bound of each wait for a peer; 0 = 2000 */
} sb_ep_desc;

#define SB_EP_HANDLE_BYTES 128

int sb_ep_create(const sb_ep_desc* desc, sb_ep** out);
int sb_ep_export(const sb_ep* h, void* handle);
int sb_ep_connect(sb_ep* h, const void* handles);
int sb_ep_connect_nccl(sb_ep* h, void* nccl_comm, void* stream);
size_t sb_ep_workspace_bytes(const sb_ep* h);
/* Expert placement (optional, the same on every rank, before a forward;
 * synchronous): perm[e] (host int32 [E], a permutation of [0,E)) is expert e's
 * position, and rank r holds the experts at positions [r*E/W, (r+1)*E/W) —
 * its local expert j being the one at position r*E/W + j, so the caller
 * passes that rank's weights in position order.  The partial sums follow the
 * tree over positions: the output equals sb_ternary_moe_swiglu on one GPU over
 * the experts in position order with ids perm[ids], bit for bit.  Spreading
 * the busy experts over the ranks evens out their GEMM work.  perm = NULL
 * restores the identity. */
int sb_ep_set_placement(sb_ep* h, const int32_t* perm);
int sb_ep_forward(sb_ep* h, const void* x, int x_dtype, int64_t batch, const int32_t* ids,
                  const float* weights, const uint32_t* gate, const uint32_t* up, const uint32_t* down,
                  const float* gate_scale, const float* up_scale, const float* down_scale,
                  void* out, int out_dtype, void* workspace, size_t workspace_bytes, void* stream);
/* Reads the handle's error word (synchronous): SB_OK, SB_ERR_DEVICE_TIMEOUT
 * (a wait for a peer ran out) or SB_ERR_INVALID (an expert id out of range). */
int sb_ep_status(sb_ep* h);
/* Failure injection for tests: one bounded wait, on this rank's GPU, for a
 * flag value no rank ever writes; sb_ep_status then reports the timeout. */
int sb_ep_inject_stale_wait(sb_ep* h, void* stream);
int sb_ep_destroy(sb_ep* h);

/* NCCL bootstrap for C callers without a communicator of their own (NCCL is
 * loaded at run time from libnccl.so.2): a 128-byte unique id made on one
 * rank and shared by the caller, then one communicator per rank. */
int sb_nccl_unique_id(void* id);
int sb_nccl_comm_init(int nranks, int rank, const void* id, void** comm);
int sb_nccl_comm_destroy(void* comm);

/* ------------------------------------------------------------------------ */
/* Enhanced BVH router (the OLMoE production router) and its top-k gate       */
/* ------------------------------------------------------------------------ */

/* EnhancedBVHRouter eval forward (python/olmoe_bvh_distill.py:422-632,
 * spectral_mode off, n_rays = 1) plus the BVHGateWrapper weight conventions
 * "softmax" and "topk_softmax" (python/olmoe_e2e_eval.py:316-971).  Replaces
 * the reference's pure-PyTorch module; the reference has no kernel for it.
 * Fixed shapes of the reference: input_proj hidden -> 512 -> 256 + LayerNorm,
 * expert head (feature + n1 + n2 + n3) -> 256 -> n1*n2*n3. */
typedef struct sb_enh sb_enh;

typedef struct {
  int hidden;        /* input_dim: multiple of 8 */
  int feature;       /* feature_dim: 32, 64 or 128 */
  int branching[3];  /* n_level1, n_level2, n_level3: each 1..32, sum <= 160 - feature,
                        product <= 256 */
} sb_enh_desc;

typedef struct {
  const float* centers;  /* [K,3] */
  const float* to3d_w;   /* [3,in] */
  const float* to3d_b;   /* [3] */
  const float* feat0_w;  /* [F,in]  feature_net.0 */
  const float* feat0_b;  /* [F] */
  const float* feat2_w;  /* [F,F]   feature_net.2 */
  const float* feat2_b;  /* [F] */
  const float* head_w;   /* [K,F+3] route_head */
  const float* head_b;   /* [K] */
} sb_enh_level;

/* Host fp32 pointers, nn.Linear layout ([out, in]); state_dict names in comments. */
typedef struct {
  const float* in0_w;   /* input_proj.0.weight [512,H] */
  const float* in0_b;   /* input_proj.0.bias   [512] */
  const float* in2_w;   /* input_proj.2.weight [256,512] */
  const float* in2_b;   /* input_proj.2.bias   [256] */
  const float* ln_w;    /* input_proj.3.weight [256] */
  const float* ln_b;    /* input_proj.3.bias   [256] */
  sb_enh_level level[3];
  const float* eh0_w;   /* expert_head.0.weight [256, F+n1+n2+n3] */
  const float* eh0_b;   /* [256] */
  const float* eh2_w;   /* expert_head.2.weight [E,256] */
  const float* eh2_b;   /* [E] */
  float temperature;    /* the module's temperature buffer */
} sb_enh_weights;

enum sb_gate_mode { SB_GATE_SOFTMAX = 0, SB_GATE_TOPK_SOFTMAX = 1, SB_GATE_HYBRID = 2 };

/* Device outputs; any pointer may be NULL (not produced). */
typedef struct {
  float* logits;        /* [B,E] the router's raw logits (_last_logits) */
  float* expert_probs;  /* [B,E] softmax(logits / max(T, 0.1)) */
  int64_t* expert_ids;  /* [B]   argmax, first index on ties */
  float* geo_dist;      /* [B,E] d1[i] + d2[j] + d3[k] (_last_geometric_distances) */
  float* branch_bonus;  /* [B,E] 1 + 0.2 same domain + 0.1 same subdomain (_last_branch_bonus) */
  float* router_probs;  /* [B,E] gate router_probs */
  float* topk_weights;  /* [B,k] gate top-k weights (fp32, before the cast to the hidden dtype) */
  int32_t* topk_ids;    /* [B,k] gate top-k ids, value order, lower index first on ties */
} sb_enh_outputs;

int sb_enh_create(const sb_enh_desc* desc, int device, sb_enh** out);
int sb_enh_upload(sb_enh* h, const sb_enh_weights* w);
size_t sb_enh_workspace_bytes(const sb_enh* h, int64_t batch, int precision);
/* x: device [B,H], SB_F32 or SB_BF16 (SB_PREC_FAST needs SB_BF16).  The gate
 * rounds the logits to round_dtype (the hidden-state dtype, SB_F32 or SB_BF16)
 * before its softmax / top-k, as the reference wrapper's logits.to(dtype). */
int sb_enh_forward(sb_enh* h, const void* x, int x_dtype, int64_t batch, int precision,
                   int gate_mode, int norm_topk_prob, int round_dtype, int top_k,
                   const sb_enh_outputs* out, void* workspace, size_t workspace_bytes, void* stream);

/* Hybrid pre-filter gate (python/olmoe_e2e_eval.py:1264-1296, the
 * _hybrid_forward that replace_gate_with_bvh(hybrid=True) installs): the BVH
 * router's expert_probs pick n_candidates experts (top-n, lower index first on
 * ties); the layer's own dense gate gives full_logits = x W_gate^T in the
 * hidden dtype and router_probs = softmax(full_logits) over all E experts in
 * fp32; the top_k of router_probs among the candidates are the outputs
 * (renormalised when norm_topk_prob).
 *
 * sb_enh_set_dense_gate copies W_gate [E, hidden] (nn.Linear layout, SB_F32 or
 * SB_BF16; host or device memory) into the handle. */
int sb_enh_set_dense_gate(sb_enh* h, const void* w_gate, int w_dtype, int rows, int cols);
/* x as for sb_enh_forward; round_dtype = the hidden dtype, applied to the dense
 * logits (the BVH probabilities are computed in fp32 as the reference does on
 * x.float()).  out->router_probs receives the full dense softmax; the other
 * router outputs (logits, expert_probs, ...) are produced as by sb_enh_forward. */
int sb_enh_forward_hybrid(sb_enh* h, const void* x, int x_dtype, int64_t batch, int precision,
                          int n_candidates, int norm_topk_prob, int round_dtype, int top_k,
                          const sb_enh_outputs* out, void* workspace, size_t workspace_bytes,
                          void* stream);
int sb_enh_destroy(sb_enh* h);

/* ------------------------------------------------------------------------ */
/* MoE pipeline stage kernels (cuda/async_pipeline.cu:79-230,                */
/* python/async_pipeline_bridge.py:89-150).  Device pointers, async on       */
/* `stream`, no handle.                                                       */
/* ------------------------------------------------------------------------ */

/* Per token: optional calibration c = W raw + b (apply_calibration_kernel,
 * async_pipeline.cu:150-170; W [E,E] nn.Linear layout, E <= 128), softmax over
 * the E values when apply_softmax (softmax_topk_kernel, :177-230), then the
 * top_k values in descending order, the lower expert index first among equal
 * values (-inf ranks last; NaN ranks as -inf and is reported as -inf).  probs [B,E] (may be NULL) receives the values ranked (calibrated /
 * softmaxed); topk_weights [B,k] (may be NULL) the chosen values, not
 * renormalised.  E <= 1024, top_k <= 32. */
int sb_softmax_topk(const float* logits, int64_t batch, int n_experts, int top_k, const float* cal_w,
                    const float* cal_b, int apply_softmax, float* probs, uint32_t* topk_ids,
                    float* topk_weights, void* stream);
/* out [B,E] = raw [B,E] W^T + b, the calibration step alone. */
int sb_apply_calibration(const float* raw, int64_t batch, int n_experts, const float* cal_w,
                         const float* cal_b, float* out, void* stream);
/* Groups the B*k routing entries by expert (scatter_by_expert_kernel,
 * async_pipeline.cu:79-101): expert_counts[e] = number of entries with id e
 * (ids >= n_experts are skipped, as the reference's sentinel); entry slots in
 * ascending entry order r = t*k + j (deterministic: the reference assigns
 * slots by atomicAdd); dispatch_indices[e * max + slot] = t (or r when
 * store_entry) for slot < max_tokens_per_expert, as the reference's limit. */
int sb_scatter_by_expert(const uint32_t* expert_ids, int64_t batch, int top_k, int n_experts,
                         int max_tokens_per_expert, int store_entry, int32_t* dispatch_indices,
                         int32_t* expert_counts, void* stream);
/* ------------------------------------------------------------------------ */
/* Legacy ray-sphere tree router (cuda/v5/bvh_router_kernel.cu:244-371, the   */
/* kernel behind the reference's ctypes library and its bvh_router_ext torch  */
/* extension, cuda/v5/bvh_torch_ext.cu:270-371).  Fixed tree: 85 nodes (root, */
/* 4, 16, 64 leaves); per level the child of least |ray - center|^2 - r^2,    */
/* the child's 3x4 portal applied to the ray; scores exp(-|ray - leaf|^2).    */
/* ------------------------------------------------------------------------ */
typedef struct sb_tree sb_tree;
int sb_tree_create(int device, sb_tree** out);
/* Host fp32: centers [85,3], radii [85], portals [85,12] (row-major 3x4);
 * snell_w [85,64] and snell_b [85] are accepted for the reference signature
 * (the dispersion they drive changes no output) and may be NULL. */
int sb_tree_upload(sb_tree* h, const float* centers, const float* radii, const float* portals,
                   const float* snell_w, const float* snell_b);
/* Device pointers: origins/directions [B,3]; outputs (any may be NULL): expert
 * [B] (leaf 0..63), scores [B,64], path [B,3] (node ids 1..84), confidence [B]. */
int sb_tree_route(sb_tree* h, const float* origins, const float* directions, int64_t batch,
                  int32_t* expert, float* scores, int32_t* path, float* confidence, void* stream);
int sb_tree_destroy(sb_tree* h);

/* The reference's ctypes ABI (cuda/v5/bvh_router_kernel.cu:378-717), same names
 * and signatures, process-global: 0 ok, -1 failure.  bvh_route_batch is
 * synchronous on host buffers; use_graph=1 replays one CUDA graph per batch
 * size (copies through pinned staging, so any caller buffers are valid). */
int bvh_upload_tree(const float* centers, const float* radii, const float* portals, const float* snell_w,
                    const float* snell_b);
int bvh_alloc_buffers(int batch_size);
void bvh_free_buffers(void);
int bvh_route_batch(const float* h_origins, const float* h_directions, const float* h_spectral, int* h_expert,
                    float* h_scores, int* h_path, float* h_confidence, int batch_size, int use_graph);
int bvh_get_batch_capacity(void);
int bvh_get_num_nodes(void);
int bvh_get_num_experts(void);
int bvh_get_spec_dim(void);

/* ------------------------------------------------------------------------ */
/* The OptiX router's route / route_topk served by CUDA                       */
/* (cuda/v5/optix_training_ext.cu:182-263; programs cuda/optix_router_raygen.cu, */
/* cuda/optix_router_hitgroup.cu; geometry cuda/optix_router_host.cpp:372-600). */
/* Experts are spheres (center, radius) drawn as octahedra (use_triangles) or  */
/* boxes; a ray's closest hit in t in [0.001, 1000] gives (expert, t), a miss  */
/* (-1, 1e30).  top_k > 1 traces the reference's fan of k rays.               */
/* ------------------------------------------------------------------------ */
typedef struct sb_gas sb_gas;
int sb_gas_create(int device, sb_gas** out);
/* Host fp32 centers [n,3], radii [n]; n <= 4096. */
int sb_gas_build(sb_gas* h, const float* centers, const float* radii, int n_experts, int use_triangles);
/* Device fp32 positions/directions [B,3]; expert_ids/distances [B] (first ray
 * of the fan when top_k > 1); topk_ids/topk_dists [B,k] may be NULL. */
int sb_gas_route(sb_gas* h, const float* positions, const float* directions, int64_t batch, int top_k,
                 int32_t* expert_ids, float* distances, int32_t* topk_ids, float* topk_dists, void* stream);
int sb_gas_destroy(sb_gas* h);

/* output [B,H] = sum_j weights[t,j] * expert_outputs[t,j,:] in slot order with
 * one fused multiply-add per term (weighted_combine_kernel, async_pipeline.cu:112-132). */
int sb_weighted_combine(const float* expert_outputs, const float* weights, int64_t batch, int hidden,
                        int top_k, float* output, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SPECTRAL_B200_H */
