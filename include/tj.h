/*
 * techjam-b200 C ABI: forward pass of the reference's fixed pre-LN Transformer
 * encoder on B200 (sm_100a).  Plain pointers and sizes only; every entry point
 * returns a TjStatus and, on failure, leaves a message for tj_last_error().
 * All device work is enqueued on the caller's stream (a cudaStream_t passed as
 * void*); nothing here allocates device memory except tj_model_create /
 * tj_model_load_* (packed weights, owned by the model).
 *
 * Reference interfaces replaced (paths inside the reference repository):
 *   tj_model_create        BaselineTransformer.__init__ / TransformerConfig
 *                          (torch_transformer_benchmark.py:29-56, 148-160) and the
 *                          candidate factory CandidateSpec.model_factory
 *                          (src/infra/candidate.py:15-39, src/dispatcher.py:267-293)
 *   tj_model_load_layer    copy_model_weights -> load_state_dict
 *   tj_model_load_final_norm   (torch_transformer_benchmark.py:203-213) plus the
 *                          packed-QKV rebuild of PackedQKVSDPASelfAttention
 *                          (src/implementations/sdpa.py:96-116)
 *   tj_forward             BaselineTransformer.forward / DispatchingTransformer.forward
 *                          (torch_transformer_benchmark.py:162-172; src/dispatcher.py:708-794)
 *   tj_prepare_mask        classify_mask / _mask_kind (src/implementations/
 *                          attention_routing.py:76-98; src/dispatcher.py:393-423),
 *                          without the host synchronisation
 *   tj_layernorm           nn.LayerNorm in BaselineTransformerBlock (:128,130,160)
 *   tj_gemm_f16            the nn.Linear projections (:72-75, 131-132) with the
 *                          fused epilogues of :118-121, 141-144
 *   tj_attention_f16       BaselineSelfAttention.forward scores/softmax/PV (:97-116)
 *                          and StridedSDPASelfAttention (src/implementations/sdpa.py:46-78)
 */
#ifndef TJ_H_
#define TJ_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TJ_API __attribute__((visibility("default")))
#else
#define TJ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum TjStatus {
  TJ_OK = 0,
  TJ_ERR_INVALID = 1,      /* bad argument (null pointer, shape mismatch, bad workspace) */
  TJ_ERR_UNSUPPORTED = 2,  /* shape outside the kernels' envelope (e.g. head_dim) */
  TJ_ERR_CUDA = 3,         /* CUDA runtime / driver error */
  TJ_ERR_DEVICE = 4,       /* a kernel's bounded wait expired; see tj_device_error */
  TJ_ERR_NO_DEVICE = 5,    /* no sm_100 device is current */
  TJ_ERR_NCCL = 6          /* NCCL missing, failed or timed out (communicator aborted) */
} TjStatus;

/* Attention evaluation route for the forward pass. */
typedef enum TjAttentionRoute {
  TJ_ROUTE_EXACT = 0, /* exact causal/padded softmax attention (flash-style) */
  TJ_ROUTE_POLY = 1,  /* guarded degree-2 polynomial route; falls back to exact
                         when the fused score-range check fails */
  TJ_ROUTE_AUTO = 2   /* poly for long causal unpadded sequences, exact otherwise */
} TjAttentionRoute;

/* Which tokens a rank holds under sequence sharding (P ranks, sequence S). */
typedef enum TjShardLayout {
  TJ_SHARD_CONTIGUOUS = 0, /* rank r: [r*S/P, (r+1)*S/P) */
  TJ_SHARD_ZIGZAG = 1      /* rank r: chunks r and 2P-1-r of S/(2P) tokens, back to
                              back -- every rank gets the same causal attention
                              work; exact route only */
} TjShardLayout;

typedef struct TjConfig {
  int d_model;
  int num_heads;
  int ffn_dim;
  int num_layers;
  int causal;       /* nonzero: causal attention */
  float layer_norm_eps; /* nn.LayerNorm default 1e-5 */
} TjConfig;

/* Device pointers to one block's FP32 parameters in nn.Linear layout
   (weight [out_features, in_features] row-major). */
typedef struct TjLayerParams {
  const float* norm1_weight;
  const float* norm1_bias;
  const float* q_weight;
  const float* q_bias;
  const float* k_weight;
  const float* k_bias;
  const float* v_weight;
  const float* v_bias;
  const float* out_weight;
  const float* out_bias;
  const float* norm2_weight;
  const float* norm2_bias;
  const float* ffn_in_weight;
  const float* ffn_in_bias;
  const float* ffn_out_weight;
  const float* ffn_out_bias;
} TjLayerParams;

typedef struct TjModel TjModel;

TJ_API int tj_version(void);
/* Message of the last failing call on this thread ("" if none). */
TJ_API const char* tj_last_error(void);

/* Creates a model on the current CUDA device; allocates its packed-weight
   buffers and its device error word. */
TJ_API int tj_model_create(const TjConfig* cfg, TjModel** out);
TJ_API int tj_model_destroy(TjModel* model);
/* Converts one block's FP32 parameters into the model's packed FP16 weights
   ([3d, d] packed QKV, [d, d], [F, d], [d, F]) and FP32 biases / norms. */
TJ_API int tj_model_load_layer(TjModel* model, int layer, const TjLayerParams* params, void* stream);
TJ_API int tj_model_load_final_norm(TjModel* model, const float* weight, const float* bias, void* stream);

/* Bytes of scratch tj_forward needs for [batch, seq_len] inputs and the given
   TjAttentionRoute (the polynomial route adds its per-chunk state snapshots
   when the shape can take it: causal, head_dim 64, seq_len a multiple of 512
   above the 4096-token exact prefix; TJ_ROUTE_AUTO only from 16384 tokens).
   The workspace must be zero-filled before its first use (afterwards
   tj_forward only ever writes finite values into it). */
TJ_API int tj_workspace_bytes(const TjModel* model, int batch, int seq_len, int route, size_t* bytes);

/* out[B,S,d] = encoder(x[B,S,d]) with the reference's padding semantics:
   valid_mask[B,S] (1 byte per token, nullable = all valid); padded output rows
   are exactly 0.  x and out are FP32 device buffers and may not alias.
   route: TjAttentionRoute. */
TJ_API int tj_forward(TjModel* model, const float* x, const uint8_t* valid_mask, float* out, int batch, int seq_len,
               int route, void* workspace, size_t workspace_bytes, void* stream);

/* Allocation-free forward (no counterpart in the reference).  Same result as
   tj_forward, but its scratch lives in a fixed device array inside this
   library (TJ_NOALLOC_SCRATCH_BYTES per device, held until process exit)
   instead of a caller workspace; for callers that cannot allocate device
   memory on their call path.  Shapes whose scratch (tj_workspace_bytes)
   exceeds the array are rejected with TJ_ERR_UNSUPPORTED.  The first call on
   a device resolves the array's device address; make that first call before
   any stream capture.  All calls share the one array: calls that overlap on
   the GPU (different streams or threads) race.  The resolved address is kept
   for the life of the device's context; after cudaDeviceReset, reload the
   library before calling this again on that device. */
#define TJ_NOALLOC_SCRATCH_BYTES (32u << 20)
TJ_API int tj_forward_noalloc(TjModel* model, const float* x, const uint8_t* valid_mask, float* out, int batch,
                              int seq_len, int route, void* stream);

/* Host <-> device copy of the valid rows of right-padded samples (no
   counterpart in the reference, whose inputs start on the device): for each
   sample b, rows [b*seq_len, b*seq_len + lengths[b]) of row_bytes each, as
   cudaMemcpyAsync calls on the stream (cudaMemcpyDefault: any direction
   under unified addressing; pinned host memory for asynchrony), one per run
   of consecutive rows.  lengths is a host array.  tj_forward never reads
   the padded rows of x when valid_mask is a right-padded prefix mask, so a
   caller holding its input in host memory uploads only these rows. */
TJ_API int tj_copy_valid_rows(void* dst, const void* src, const int* lengths, int batch, int seq_len,
                              size_t row_bytes, void* stream);

/* Reads (synchronously) and clears the model's device error word: 0 if no
   kernel's bounded wait expired since the last call, else the site code of
   the first wait that did (101-103 GEMM, 201-203 attention, 301 polynomial
   route, 900 tj_wait_selftest). */
TJ_API int tj_device_error(TjModel* model, int* code);

/* Limit of every bounded wait in this library's kernels on the current
   device, in nanoseconds of GPU global-timer time (0 restores the default,
   4 s).  Applies to kernels launched after the call, for every model and
   stream on the device.  Replaces no reference interface: the reference has
   no device-side waits (its fallback contract is src/dispatcher.py:684-706). */
TJ_API int tj_set_wait_limit(unsigned long long ns);
/* Failure-path self-test (no counterpart in the reference): one warp waits on
   a barrier that nothing completes, through the same bounded wait every
   kernel uses; after the wait limit it records site code 900 in the model's
   error word (model non-null) or in *err, and returns.  Nothing faults, traps
   or hangs; the context stays usable. */
TJ_API int tj_wait_selftest(TjModel* model, int* err, void* stream);

/* Programmatic dependent launch in tj_forward (no counterpart in the
   reference): -1 = by size (on for batch*seq_len*d_model <= 2^24, where
   kernels are short enough that overlapping each one's launch and prologue
   with its predecessor's tail pays), 0 = never, 1 = always.  The initial
   mode is TJ_PDL from the environment (unset: -1).  Process-wide; changes
   no result bit. */
TJ_API int tj_set_pdl(int mode);

/* ---- per-kernel timing (CUDA events recorded around each launch) ------- */

typedef enum TjKernelClass {
  TJ_K_PREP = 0,      /* mask -> lengths / live tiles */
  TJ_K_LN = 1,        /* LayerNorm -> fp16 GEMM operand */
  TJ_K_QKV = 2,       /* packed QKV GEMM (+ head scatter) */
  TJ_K_ATTN = 3,      /* flash attention */
  TJ_K_OUT = 4,       /* output projection GEMM (+ residual) */
  TJ_K_FFN_IN = 5,    /* FFN-in GEMM (+ GELU) */
  TJ_K_FFN_OUT = 6,   /* FFN-out GEMM (+ residual) */
  TJ_K_LN_FINAL = 7,  /* final LayerNorm (fp32 out) */
  TJ_K_POLY = 8,      /* polynomial-route kernels */
  TJ_K_COUNT = 9
} TjKernelClass;

/* Start recording a CUDA-event pair around each of the next (at most)
   max_launches kernel launches of this model. */
TJ_API int tj_profile_begin(TjModel* model, int max_launches);
/* Synchronises on the recorded events and writes, per TjKernelClass, the
   summed device milliseconds and launch counts (arrays of TJ_K_COUNT). */
TJ_API int tj_profile_end(TjModel* model, double* ms_by_class, long long* launches_by_class);
/* Launches recorded while the stream was being captured into a CUDA graph
   become event-record nodes that every replay records again.  After each
   replay, this ADDS the replay's per-class milliseconds and launch counts to
   the arrays, keeping the recording (finish with tj_profile_end). */
TJ_API int tj_profile_collect(TjModel* model, double* ms_by_class, long long* launches_by_class);
/* Total kernels this model has launched (all classes, profiling or not). */
TJ_API int tj_launch_count(TjModel* model, long long* count);

/* ---- building blocks (same kernels the forward uses) ------------------- */

/* lengths[b] = 1 + last valid position; general[b] = mask is not a prefix;
   tile_list / n_live / tile_live describe the 128-row tiles of the flattened
   [B*S] rows that hold at least one valid row.  mask may be null. */
TJ_API int tj_prepare_mask(const uint8_t* mask, int batch, int seq_len, int* lengths, uint8_t* general, int* tile_list,
                    int* n_live, uint8_t* tile_live, void* stream);

/* Row-wise LayerNorm of x[rows, d] (FP32) into out (FP16 if out_fp16 else
   FP32); rows outside the valid prefix (lengths/mask, rows = batch*seq_len)
   are written as zeros (FP32 output: all of them; FP16: those in live tiles). */
TJ_API int tj_layernorm(const float* x, const float* gamma, const float* beta, int batch, int seq_len, int d, float eps,
                 void* out, int out_fp16, const int* lengths, const uint8_t* mask, const uint8_t* tile_live,
                 void* stream);

typedef enum TjEpilogue {
  TJ_EPI_QKV = 0,     /* scatter bias-added fp16 columns into Q,K,V [B,H,S,hd] */
  TJ_EPI_GELU = 1,    /* out16 = gelu_erf(acc + bias) */
  TJ_EPI_RESID = 2,   /* out32 = resid + acc + bias (resid may alias out32) */
  TJ_EPI_PLAIN16 = 3  /* out16 = acc + bias */
} TjEpilogue;

/* C[M,N] = A[M,K] (fp16, row-major) x W[N,K]^T (fp16, row-major) on tcgen05
   with fp32 accumulation, over the live 128-row tiles of tile_list; invalid
   rows (lengths/mask over rows = batch*seq_len) are written as zeros. */
TJ_API int tj_gemm_f16(const void* a, const void* w, const float* bias, int batch, int seq_len, int n, int k, int epilogue,
                void* out, const float* resid, void* q, void* k_out, void* v, int heads, const int* tile_list,
                const int* n_live, const int* lengths, const uint8_t* mask, int* err, void* stream);

/* ctx[B*S, H*hd] (fp16) = softmax(Q K^T * hd^-0.5 [+ causal/padding masks]) V
   with Q,K,V fp16 [B,H,S,hd]; hd in {32, 64, 128}.  sched (nullable): two
   zero-filled ints through which the head_dim <= 64 kernel's CTAs claim work
   items heavy-first; the kernel leaves them zero again.  Null: a static
   round-robin assignment of the same items. */
TJ_API int tj_attention_f16(const void* q, const void* k, const void* v, void* ctx, int batch, int heads, int seq_len,
                     int head_dim, int causal, const int* lengths, const uint8_t* mask, const uint8_t* general,
                     int* err, int* sched, void* stream);

/* The attention of one sequence shard, as tj_forward_seqshard runs it after
   its K/V all-gather (no counterpart in the reference; exposed so the shard
   layouts can be checked on one GPU): causal, unpadded; q is shard `rank`'s
   queries fp16 [B,H,seq_local,hd] in local row order, k_all / v_all hold
   every shard's keys / values [world][B][H][seq_local][hd], lengths[b] = the
   global sequence length, layout a TjShardLayout; ctx as tj_attention_f16. */
TJ_API int tj_attention_shard_f16(const void* q, const void* k_all, const void* v_all, void* ctx, int batch,
                                  int heads, int seq_local, int head_dim, const int* lengths, const uint8_t* general,
                                  int* err, int* sched, int rank, int world, int layout, void* stream);

/* ---- sequence sharding over NCCL (one process per GPU) ----------------- */

typedef struct TjComm TjComm;
/* 128-byte NCCL unique id, made on one rank and shared with the others by the
   host (e.g. a torch.distributed broadcast). */
TJ_API int tj_nccl_unique_id(void* id_out);
/* Joins the communicator (non-blocking NCCL init polled up to timeout_ms; on
   expiry the communicator is aborted and TJ_ERR_NCCL returned). */
TJ_API int tj_comm_create(const void* id, int rank, int world, int timeout_ms, TjComm** out);
TJ_API int tj_comm_destroy(TjComm* comm);
TJ_API int tj_workspace_bytes_seqshard(const TjModel* model, const TjComm* comm, int batch, int seq_local, int route,
                                       size_t* bytes);
/* Forward of rank r's sequence shard: x/out hold rank r's tokens of every
   sample ([B, seq_local, d], FP32, causal, no padding) -- global tokens
   [r*seq_local, (r+1)*seq_local) for TJ_SHARD_CONTIGUOUS, or the chunks
   [r*h, (r+1)*h) and [(2P-1-r)*h, (2P-r)*h), h = seq_local/2, in that order
   for TJ_SHARD_ZIGZAG (route TJ_ROUTE_EXACT only, seq_local a multiple of
   512).  Token-local work runs on the shard; attention takes
   the guarded polynomial route (guard statistics all-reduced so every rank
   decides alike; each rank's state total all-gathered and folded into its
   snapshots) or the exact flash route over all-gathered K/V.  The guard runs
   on the first forward of a shard shape (batch, seq_local, world), with one
   host read of its verdict per layer; later forwards reuse each layer's
   verdict and coefficients without guard kernels or host synchronisation, as
   the reference estimates sigma once per attention module and caches it
   (src/implementations/extreme.py:297-301).  Reloading a layer's weights
   re-evaluates it; every rank must do so alike.  Replaces the single-GPU
   prefix streaming of forward_prefix_chunks
   (src/implementations/extreme.py:167-204). */
TJ_API int tj_forward_seqshard(TjModel* model, TjComm* comm, const float* x, float* out, int batch, int seq_local,
                               int route, int layout, void* workspace, size_t workspace_bytes, void* stream);
/* The sequence-sharded guard's cached verdict for a layer: 1 polynomial
   route, 0 exact route, -1 not evaluated yet (no counterpart in the
   reference beyond PolyOrFlashSelfAttention.route_name, extreme.py:268-272). */
TJ_API int tj_seqshard_route(const TjModel* model, int layer, int* route);

/* Guarded polynomial causal attention over Q,K,V fp16 [B,H,S,64] with no
   padding (lengths[b] == S), replacing PolyOrFlashSelfAttention.forward +
   poly_attention_forward (src/implementations/extreme.py:276-319,
   poly_attention.py:21-83; algorithm poly_reference.py:61-265; guard
   poly_guard.py:65-102): a device-side score-range check admits the route
   (sigma <= 0.40, max |s| <= 10, unpadded); queries < exact_prefix, or all of
   them when not admitted, take the exact flash kernel.  The workspace starts
   with a TjPolyStatus describing the last call. */
typedef struct TjPolyStatus {
  int admit;             /* 1 = polynomial route ran, 0 = exact fallback */
  float c0, c1, c2;      /* Hermite coefficients used */
  float sigma;           /* std of the sampled scaled scores */
  float max_abs;         /* max |scaled score| in the sample */
} TjPolyStatus;
TJ_API int tj_poly_workspace_bytes(int batch, int heads, int seq_len, int exact_prefix, size_t* bytes);
TJ_API int tj_poly_attention_f16(const void* q, const void* k, const void* v, void* ctx, const int* lengths,
                                 int batch, int heads, int seq_len, int exact_prefix, void* workspace,
                                 size_t workspace_bytes, int* err, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* TJ_H_ */
