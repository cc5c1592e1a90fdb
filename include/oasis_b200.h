/*
 * oasis_b200.h - C ABI of the B200 (sm_100a) Oasis-500M frame-generation library.
 *
 * One frame = 4 DDIM v-prediction steps through the 16-block spatio-temporal DiT,
 * then the 12-block ViT VAE decode. The functions below are what a host binding
 * (ctypes here; cgo/JNI/N-API elsewhere) calls in place of the reference's device
 * code in zoecarver/open-oasis `oasis_inference.py`.
 *
 * Conventions
 *   - All pointers are caller-owned DEVICE pointers. Tensors marked bf16 hold
 *     IEEE bfloat16 (uint16 storage); everything else is fp32. Row-major.
 *   - The library never allocates on these paths: scratch comes from a caller
 *     workspace sized by the matching *_workspace_size() function.
 *   - Every call is stream-ordered on `stream` (a cudaStream_t; NULL = legacy
 *     default stream) and returns 0 or a negative OASIS_ERR_* code; the reason is
 *     in oasis_last_error(). Nothing exits, traps or prints.
 *   - Kernels never spin forever: a wait that exceeds its limit sets a device
 *     error word (oasis_device_error) and the kernel returns.
 *
 * Model constants: D = 1024, 16 heads x 64, MLP 4096, 144 tokens per frame
 * (9 x 16 patches of 2 x 2 over a 16 x 18 x 32 latent), VAE 576 tokens (18 x 32)
 * decoding 20 x 20 x 3 pixel patches into a 3 x 360 x 640 frame.
 */
#ifndef OASIS_B200_H
#define OASIS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* oasis_stream_t; /* cudaStream_t */

#define OASIS_OK 0
#define OASIS_ERR_INVALID_ARG (-1)
#define OASIS_ERR_CUDA (-2)
#define OASIS_ERR_WORKSPACE (-3)
#define OASIS_ERR_DEVICE_TIMEOUT (-4)
#define OASIS_ERR_UNSUPPORTED (-5)

#define OASIS_DIT_SUBBLOCKS 32       /* blocks.{0..15}.{s,t} interleaved: 2i = spatial, 2i+1 = temporal */
#define OASIS_ADALN_WIDTH 6144       /* per sub-block adaLN output (shift, 1+scale, gate) x (msa, mlp) */
#define OASIS_ADALN_ROWS (OASIS_DIT_SUBBLOCKS * OASIS_ADALN_WIDTH + 2048) /* + final (shift, 1+scale) */
#define OASIS_MAX_FRAMES 32          /* temporal positions of rope_temporal (T <= 32) */
#define OASIS_VAE_BLOCKS 12          /* max ViT blocks of the VAE decoder and of its encoder */
#define OASIS_VAE_ENC_K 1216         /* patch_embed GEMM depth: 3 x 20 x 20 = 1200 pixels, zero-padded to 19 x 64 */

/* ---------------------------------------------------------------- errors -- */

/* Message of the last failing call on this host thread ("" if none). */
const char* oasis_last_error(void);
/* The same message under the name the boundary specification uses. */
const char* oasis_get_last_error(void);
/* Reads (and with reset != 0 clears) the device error word; synchronizes the device. */
int oasis_device_error(int reset);
/* Number of kernels this library has launched from the host so far (graph
 * replays launch without the host and are not counted). */
unsigned long long oasis_launch_count(void);
/* Library version string. */
const char* oasis_version(void);

/* ------------------------------------------------------------- weights --- */

/* One DiT sub-block (blocks.i.s or blocks.i.t). Replaces the per-prefix device
 * tensors of preload_dit_weights (oasis_inference.py:546-626): the reference's
 * [Q|K|V|Qswap|Kswap] packing is unnecessary because RoPE is applied in the QKV
 * GEMM epilogue. Weights keep the nn.Linear [out, in] layout. */
typedef struct OasisDitSubBlock {
  const void* qkv_w;  /* bf16 [3072, 1024], no bias (to_qkv) */
  const void* out_w;  /* bf16 [1024, 1024] (to_out) */
  const float* out_b; /* [1024] */
  const void* fc1_w;  /* bf16 [4096, 1024] */
  const float* fc1_b; /* [4096] */
  const void* fc2_w;  /* bf16 [1024, 4096] */
  const float* fc2_b; /* [1024] */
} OasisDitSubBlock;

typedef struct OasisDitWeights {
  int num_subblocks; /* 32 for Oasis-500M; fewer runs a truncated stack (tests) */
  OasisDitSubBlock sub[OASIS_DIT_SUBBLOCKS];
  /* All sub-block adaLN linears plus the final layer's, stacked along the
   * output dim: rows [6144 i, 6144 i + 6144) = blocks.(i/2).(s|t)_adaLN_modulation.1,
   * rows [6144 S, 6144 S + 2048) = final_layer.adaLN_modulation.1 (S = num_subblocks).
   * Bias has +1 folded into every scale slice (oasis_inference.py:549-556, 531). */
  const void* adaln_w;  /* bf16 [6144 S + 2048, 1024] */
  const float* adaln_b; /* [6144 S + 2048] */
  const void* final_w;  /* bf16 [64, 1024] final_layer.linear */
  const float* final_b; /* [64] */
  /* x_embedder conv 2x2/2 as a linear map over a (p, q, c)-ordered 64-vector
   * (W_rt of oasis_inference.py:1821-1826), stored input-major: [64, 1024]. */
  const float* embed_w; /* [64, 1024] */
  const float* embed_b; /* [1024] */
  /* RoPE tables as (cos, sin) pairs per position and head-dim pair. */
  const float* rope_spatial;  /* [16, 144, 4] axial (h, w): (cos, sin) of pairs 2q, 2q+1 at [q, pos] */
  const float* rope_temporal; /* [16, 32, 4]  frame index t < 32, same layout */
} OasisDitWeights;

typedef struct OasisVaeBlock {
  const float* norm1_w; const float* norm1_b; /* [1024] */
  const void* qkv_w; const float* qkv_b;      /* bf16 [3072, 1024], [3072] */
  const void* proj_w; const float* proj_b;    /* bf16 [1024, 1024], [1024] */
  const float* norm2_w; const float* norm2_b; /* [1024] */
  const void* fc1_w; const float* fc1_b;      /* bf16 [4096, 1024], [4096] */
  const void* fc2_w; const float* fc2_b;      /* bf16 [1024, 4096], [1024] */
} OasisVaeBlock;

typedef struct OasisVaeWeights {
  const float* post_quant_w; /* [16, 1024] input-major (post_quant_conv as a linear map) */
  const float* post_quant_b; /* [1024] */
  int num_blocks;            /* 12 for Oasis-500M's decoder; fewer in tests */
  OasisVaeBlock blk[OASIS_VAE_BLOCKS];
  const float* norm_w; const float* norm_b; /* dec_norm [1024] */
  const void* pred_w;                       /* bf16 [1200, 1024] predictor */
  const float* pred_b;                      /* [1200] */
  const float* rope;                        /* [16, 576, 4] as rope_spatial; pairs >= 16 are (1, 0) */
} OasisVaeWeights;

/* VAE encoder weights (the `encoder.*` half of the VAE checkpoint that
 * oasis_inference.py:499-503 locates; used by vae.encode at :1744-1756).
 * Layout: patch_embed conv 20x20/20 (3 -> 1024) as a GEMM over each patch's
 * (c, p, q)-ordered 1200 pixels, num_blocks pre-LN ViT blocks with the same
 * structure, pixel RoPE and GELU as the decoder's, the final LayerNorm, then
 * quant_conv (1024 -> 32: posterior mean | logvar). */
typedef struct OasisVaeEncoderWeights {
  const void* patch_w;    /* bf16 [1024, OASIS_VAE_ENC_K] (conv weight flattened, zero-padded 1200 -> K) */
  const float* patch_b;   /* [1024] */
  int num_blocks;         /* depth of the encoder (from the checkpoint's encoder.* keys) */
  OasisVaeBlock blk[OASIS_VAE_BLOCKS];
  const float* norm_w; const float* norm_b; /* final encoder LayerNorm [1024] */
  const void* quant_w;                      /* bf16 [32, 1024] */
  const float* quant_b;                     /* [32] */
  const float* rope;                        /* [16, 576, 4], as OasisVaeWeights.rope */
} OasisVaeEncoderWeights;

/* Conditioning weights (t_embedder and external_cond of the DiT checkpoint), fp32,
 * nn.Linear [out, in] layout. Replaces the host copies compute_cond_for_frame
 * reads (dev["t_emb_w0_host"] etc., oasis_inference.py:1406-1427). */
typedef struct OasisCondWeights {
  const float* t_freqs;             /* [128] exp(-ln(10000) i / 128), the timestep embedding frequencies */
  const float* t_w0; const float* t_b0; /* [1024, 256], [1024] t_embedder.mlp.0 */
  const float* t_w2; const float* t_b2; /* [1024, 1024], [1024] t_embedder.mlp.2 */
  const float* ext_w; const float* ext_b; /* [1024, 25], [1024] external_cond (may be NULL without actions) */
} OasisCondWeights;

/* ---------------------------------------------------------- composite ---- */

/* DiT forward over B sessions x T frames (T <= 32).
 * Replaces dit_forward_device (oasis_inference.py:1438-1526).
 *   z     [B, T, 144, 1024] fp32 token embeddings; used as the residual stream
 *         and overwritten.
 *   cond  [B, T, 1024] fp32 conditioning per frame (before SiLU).
 *   v_out last_frame_only ? [B, 144, 64] : [B, T, 144, 64] fp32 v-prediction. */
typedef struct OasisDitArgs {
  int batch;
  int frames;
  float* z;
  const float* cond;
  float* v_out;
  int last_frame_only;
  void* workspace;
  size_t workspace_bytes;
} OasisDitArgs;

size_t oasis_dit_workspace_size(int batch, int frames);
int oasis_dit_forward(const OasisDitWeights* w, const OasisDitArgs* a, oasis_stream_t stream);

/* DDIM coefficients of one step (oasis_inference.py:1843-1860):
 * x0 = at_sqrt x - one_minus_at_sqrt v; eps = (inv_at_sqrt x - x0) inv_sigma;
 * x' = an_sqrt x0 + one_minus_an_sqrt eps. */
typedef struct OasisDdimCoeffs {
  float at_sqrt, one_minus_at_sqrt, inv_at_sqrt, inv_sigma, an_sqrt, one_minus_an_sqrt;
} OasisDdimCoeffs;

/* In-place DDIM update of n elements. Replaces the eltwise tail of ddim_step_fn
 * (oasis_inference.py:1920-1931). */
int oasis_ddim_update(float* chunk, const float* v, const OasisDdimCoeffs* c, long long n,
                      oasis_stream_t stream);

/* One full DDIM step (ddim_step_fn, oasis_inference.py:1909-1932):
 * z = concat(context_z, patch_embed(chunk)); v = DiT(z, cond)[last frame];
 * chunk = ddim(chunk, v).
 *   chunk     [B, 144, 64] fp32 noisy latent patches, (p, q, c) order; updated in place
 *   context_z [B, T-1, 144, 1024] fp32 embedded context frames (may be NULL if T == 1)
 *   cond      [B, T, 1024] fp32 */
typedef struct OasisStepArgs {
  int batch;
  int frames;
  float* chunk;
  const float* context_z;
  const float* cond;
  OasisDdimCoeffs coeffs;
  void* workspace;
  size_t workspace_bytes;
} OasisStepArgs;

size_t oasis_step_workspace_size(int batch, int frames);
int oasis_ddim_step(const OasisDitWeights* w, const OasisStepArgs* a, oasis_stream_t stream);

/* Patch-embed latent patches [rows, 64] into token rows of z:
 * out_row = (r / 144) * out_group + out_off + r % 144. */
int oasis_patch_embed(const OasisDitWeights* w, const float* patches, int rows, float* z,
                      long long out_group, long long out_off, oasis_stream_t stream);

/* DiT output chunk [B, 144, 64] -> VAE latent tokens [B, 576, 16] scaled by
 * 1 / 0.07843137255. Replaces bridge_unpatchify (oasis_inference.py:1697-1709). */
int oasis_bridge_unpatchify(const float* chunk, float* latent, int batch, oasis_stream_t stream);

/* VAE decode of B frames. Replaces vae_decode_forward (oasis_inference.py:1546-1618)
 * plus vae_unpatchify and the clamp (oasis_inference.py:1636-1645, 2292).
 *   latent [B, 576, 16] fp32 (already divided by the scaling factor)
 *   image  [B, 3, 360, 640] fp32 clamped to [-1, 1] */
typedef struct OasisVaeArgs {
  int batch;
  const float* latent;
  float* image;
  void* workspace;
  size_t workspace_bytes;
} OasisVaeArgs;

size_t oasis_vae_workspace_size(int batch);
int oasis_vae_decode(const OasisVaeWeights* w, const OasisVaeArgs* a, oasis_stream_t stream);

/* VAE encode of B prompt images. Replaces `vae.encode(x).mean * SCALING_FACTOR`
 * (oasis_inference.py:1748-1751) and the patch re-layout before the context
 * patch embed (:1752-1754, 1806-1809).
 *   image  [B, 3, 360, 640] fp32 in [-1, 1]
 *   latent [B, 576, 16] fp32 posterior mean x 0.07843137255 (may be NULL)
 *   chunk  [B, 144, 64] fp32 the same latent in the DiT's (p, q, c) patch layout,
 *          ready for oasis_patch_embed (may be NULL; not both) */
typedef struct OasisVaeEncodeArgs {
  int batch;
  const float* image;
  float* latent;
  float* chunk;
  void* workspace;
  size_t workspace_bytes;
} OasisVaeEncodeArgs;

size_t oasis_vae_encoder_workspace_size(int batch);
int oasis_vae_encode(const OasisVaeEncoderWeights* w, const OasisVaeEncodeArgs* a, oasis_stream_t stream);

/* One generated frame for B sessions (run_full_frame, oasis_inference.py:2175-2232):
 * `steps` DDIM steps through the DiT, then the bridge and the VAE decode. The
 * adaLN tables of all steps come from one GEMM, so the stacked adaLN weights are
 * read once per frame instead of once per step.
 *   chunk     [B, 144, 64] fp32 noise patches in, final latent patches out
 *   context_z [B, T-1, 144, 1024] fp32 embedded context frames (NULL if T == 1)
 *   cond      [steps, B, T, 1024] fp32 conditioning of every step (pre-SiLU)
 *   coeffs    HOST array of `steps` DDIM coefficient sets, highest noise first
 *   image     [B, 3, 360, 640] fp32 in [-1, 1]; skip_decode != 0 stops after the steps */
typedef struct OasisFrameArgs {
  int batch;
  int frames;
  int steps;
  float* chunk;
  const float* context_z;
  const float* cond;
  const OasisDdimCoeffs* coeffs;
  float* image;
  int skip_decode;
  void* workspace;
  size_t workspace_bytes;
} OasisFrameArgs;

size_t oasis_frame_workspace_size(int batch, int frames, int steps);
int oasis_generate_frame(const OasisDitWeights* w, const OasisVaeWeights* vw, const OasisFrameArgs* a,
                         oasis_stream_t stream);

/* Frame conditioning on the GPU, fp32 (compute_cond_for_frame,
 * oasis_inference.py:1406-1427, which the reference runs on the host):
 *   cond[r] = t_mlp([cos(t f) | sin(t f)], t = levels[r])
 *             + (actions ? actions[r % action_rows] . ext_w^T + ext_b : 0)
 *   levels  [n] fp32 noise levels (integers as floats), device
 *   actions [action_rows, 25] fp32 or NULL; row r uses actions[r % action_rows],
 *           so a [B, T, 25] action window serves rows laid out [S][B][T]
 *   cond    [n, 1024] fp32
 * Workspace: oasis_cond_workspace_size(n) bytes (the hidden layer). */
size_t oasis_cond_workspace_size(int n);
int oasis_compute_cond(const OasisCondWeights* w, const float* levels, int n, const float* actions, int action_rows,
                       float* cond, void* workspace, size_t workspace_bytes, oasis_stream_t stream);

/* ---------------------------------------------------- context caching --- */
/* The context frames attend only to earlier frames (causal temporal attention)
 * and keep the same conditioning at every DDIM step, so their rows can be run
 * once per generated frame and only the generated frame's rows per step
 * (oasis_inference.py:1218-1403, default path :1934-1960; the reference does
 * this for one context frame, here for any T - 1 <= 31).
 *
 * KV cache: for each of the 16 temporal sub-blocks, the packed RoPE'd QKV rows
 * of the context frames, bf16 [16][B, T-1, 144, 3072]. */
size_t oasis_kv_cache_size(int batch, int past_frames);

/* Replaces precompute_past_state (oasis_inference.py:1354-1369). a->frames =
 * T - 1 context frames; a->z [B, T-1, 144, 1024] fp32 is overwritten; a->cond
 * [B, T-1, 1024]; a->v_out is not used. Workspace: oasis_dit_workspace_size(B, T-1). */
int oasis_dit_precompute_past(const OasisDitWeights* w, const OasisDitArgs* a, void* kv_cache, size_t kv_cache_bytes,
                              oasis_stream_t stream);

/* Replaces dit_forward_currentonly (oasis_inference.py:1372-1403). a->frames = 1;
 * a->z [B, 144, 1024] fp32 generated frame (overwritten); a->cond [B, 1024];
 * a->v_out [B, 144, 64]. The generated frame sits at temporal position
 * past_frames. Workspace: oasis_dit_workspace_size(B, 1). */
int oasis_dit_forward_current(const OasisDitWeights* w, const OasisDitArgs* a, const void* kv_cache,
                              size_t kv_cache_bytes, int past_frames, oasis_stream_t stream);

/* oasis_generate_frame with the context rows run once (same arguments and
 * results up to rounding; the KV cache lives in the workspace). */
size_t oasis_frame_kv_workspace_size(int batch, int frames, int steps);
int oasis_generate_frame_kv(const OasisDitWeights* w, const OasisVaeWeights* vw, const OasisFrameArgs* a,
                            oasis_stream_t stream);

/* ---------------------------------------------------- tensor parallelism --- */
/* n-way tensor parallelism of the DiT forward (the reference's multi-chip scheme,
 * oasis_inference.py:289-305, 569-626, 1153-1201). `shard` holds this rank's
 * slices: for its heads = 16 / n heads (HD = 64 heads columns) qkv_w [3 HD, 1024]
 * (its q, k and v rows), out_w [1024, HD], fc1_w [4 HD, 1024] + fc1_b [4 HD],
 * fc2_w [1024, 4 HD]; out_b, fc2_b, adaLN, final layer, embed and RoPE are the
 * full (replicated) tensors. After each row-parallel projection (O, FC2) the fp32
 * partial [B T 144, 1024] in `partial` is summed over the ranks by the caller's
 * `allreduce` (issued in order on `stream`: ncclAllReduce, torch.distributed, a
 * peer-memory kernel), then bias, gate and residual are applied. z, cond and
 * v_out are replicated and have the oasis_dit_forward layouts (v_out: last
 * frame). Returns the first non-zero status of a kernel or of `allreduce`. */
typedef int (*oasis_allreduce_fn)(float* buf, size_t count, void* user, oasis_stream_t stream);

typedef struct OasisTpArgs {
  int batch;
  int frames;
  int heads;         /* this rank's heads: 16 / n */
  float* z;          /* [B, T, 144, 1024] fp32, overwritten */
  const float* cond; /* [B, T, 1024] */
  float* v_out;      /* [B, 144, 64] */
  float* partial;    /* [B T 144, 1024] fp32, the collective's buffer */
  oasis_allreduce_fn allreduce;
  void* allreduce_user;
  void* workspace;
  size_t workspace_bytes;
} OasisTpArgs;

size_t oasis_tp_workspace_size(int batch, int frames, int heads);
int oasis_dit_forward_tp(const OasisDitWeights* shard, const OasisTpArgs* a, oasis_stream_t stream);

/* Sequence-parallel form of the same n-way tensor parallelism (Megatron-style):
 * the residual stream stays sharded by session - rank r owns sessions
 * [r B / n, (r + 1) B / n) - so LayerNorm, adaLN and the gated residuals run on
 * 1/n of the rows. Per sub-block the collectives are an all-gather of the
 * LayerNorm output (bf16) before each column-parallel projection (QKV, FC1) and a
 * reduce-scatter of the row-parallel partials (O, FC2) back to the owned rows,
 * in place of the all-reduce: half the bytes at fp32 partials, a quarter at bf16.
 * Same weight shards as oasis_dit_forward_tp. Replaces the same reference code
 * (oasis_inference.py:289-305, 1153-1201).
 *
 * Collective callbacks, issued in order on `stream` (NCCL, torch.distributed,
 * a peer-memory kernel); `count` is elements per rank, `dtype` an OASIS_DTYPE_*:
 *   reduce_scatter: recv[i] = sum over ranks k of send_k[rank count + i]
 *                   (send: world x count, recv: count)
 *   all_gather:     recv[k count + i] = send_k[i] (send: count, recv: world x count)
 * A non-zero return aborts the forward with that status. The communication
 * buffers are caller-owned so the callbacks can name them. */
#define OASIS_DTYPE_F32 0
#define OASIS_DTYPE_BF16 1
typedef int (*oasis_collective_fn)(const void* send, void* recv, size_t count, int dtype, void* user,
                                   oasis_stream_t stream);

typedef struct OasisTpSpArgs {
  int batch;          /* B sessions over all ranks; B % world == 0 */
  int frames;         /* T <= 32 */
  int heads;          /* this rank's heads: 16 / world */
  int rank, world;
  float* z;           /* [B / world, T, 144, 1024] fp32: this rank's sessions, overwritten */
  const float* cond;  /* [B / world, T, 1024] */
  float* v_out;       /* [B, 144, 64] fp32: the last frame of every session (gathered) */
  int partial_dtype;  /* OASIS_DTYPE_BF16 or OASIS_DTYPE_F32: type of partial / shard */
  void* partial;      /* [B T 144, 1024] partial_dtype: row-parallel output, reduce_scatter send */
  void* shard;        /* [B T 144 / world, 1024] partial_dtype: reduce_scatter recv */
  void* xn_local;     /* [B T 144 / world, 1024] bf16: LayerNorm of the owned rows, all_gather send */
  void* xn;           /* [B T 144, 1024] bf16: all_gather recv, the projections' input */
  float* v_local;     /* [B / world, 144, 64] fp32: all_gather send of v_out */
  oasis_collective_fn reduce_scatter;
  oasis_collective_fn all_gather;
  void* user;
  void* workspace;
  size_t workspace_bytes;
  /* Overlap (optional): with comm_stream non-NULL the collectives are issued on
   * comm_stream (the callbacks receive it as `stream`) and each rank's sessions
   * are processed in `chunks` groups (chunks divides B / world, at most 8), so
   * the all-gather / reduce-scatter of one group runs while the projections of
   * the next compute; the library orders the two streams with events and
   * returns with `stream` waiting for the last collective. NULL / chunks <= 1:
   * everything in order on `stream`. */
  oasis_stream_t comm_stream;
  int chunks;
  /* With comm_stream: SMs the GEMM and attention kernels leave free so that the
   * collective kernels (NCCL's run on SMs) can execute beside them; 0 = none. */
  int reserve_sms;
} OasisTpSpArgs;

size_t oasis_tp_sp_workspace_size(int batch, int frames, int heads, int world);
int oasis_dit_forward_tp_sp(const OasisDitWeights* shard, const OasisTpSpArgs* a, oasis_stream_t stream);

/* Peer-memory collectives over NVLink (an alternative to NCCL behind the same
 * two callbacks; replaces the reference's multi-chip all-reduce,
 * oasis_inference.py:1153-1201, on the mesh of :289-305). The bulk data moves
 * on the copy engines (cudaMemcpyAsync into a peer's buffer opened through CUDA
 * IPC); these entry points carry the rest:
 *   oasis_peer_alloc / free:      device memory that can be shared by IPC (zeroed)
 *   oasis_ipc_get / open / close: the CUDA IPC handle of such an allocation
 *   oasis_peer_copy:   cudaMemcpyAsync (unified addressing) on `stream`: over
 *       NVLink on the copy engines when dst or src is a peer's memory
 *   oasis_peer_signal: one thread stores `value` to `flag` (this GPU's memory or
 *       a peer's, release at system scope) after the work before it on `stream`
 *   oasis_peer_wait:   waits on `stream` until flags[i] >= target for every
 *       i < n except `skip` (acquire, system scope); after timeout_ns it gives
 *       up, records a device error (oasis_device_error() returns 16) and returns
 *   oasis_reduce_slots: dst[i] = sum over k < n, in rank order and in fp32, of
 *       slot_k[i], slot_k = staging + k slot_stride (elements) except
 *       slot own_slot = own; written in `dtype` (count, slot_stride multiples of 8) */
#define OASIS_IPC_HANDLE_BYTES 64
int oasis_peer_alloc(size_t bytes, void** ptr);
int oasis_peer_free(void* ptr);
int oasis_ipc_get_handle(void* ptr, void* handle_out);
int oasis_ipc_open_handle(const void* handle, void** ptr);
int oasis_ipc_close_handle(void* ptr);
int oasis_peer_copy(void* dst, const void* src, size_t bytes, oasis_stream_t stream);
int oasis_peer_signal(int* flag, int value, oasis_stream_t stream);
int oasis_peer_wait(const int* flags, int n, int skip, int target, long long timeout_ns, oasis_stream_t stream);
int oasis_reduce_slots(void* dst, const void* staging, long long slot_stride, const void* own, int own_slot, int n,
                       long long count, int dtype, oasis_stream_t stream);

/* ------------------------------------------------------------ op level --- */

/* tcgen05 GEMM: acc = A[M,K] . W[N,K]^T (bf16 in, fp32 accumulate) + bias, then
 * the fused epilogue `mode`:
 *   0 F32          out_f32 = acc
 *   1 BF16         out_bf16 = acc
 *   2 GELU_TANH    out_bf16 = gelu_tanh(acc)          (DiT FC1, ttnn.linear gelu)
 *   3 GELU_ERF     out_bf16 = gelu_erf(acc)           (VAE FC1)
 *   4 GATED_RESID  out_f32 = resid + gate[r / rows_per_frame, n] * acc   (O / FC2)
 *   5 RESID        out_f32 = resid + acc              (VAE proj / FC2)
 *   6 ROPE         out_bf16 = acc with interleaved RoPE on columns [0, 2 rope_dim)
 *                  at position (r / rope_div) % rope_mod    (QKV + rope_layout);
 *                  rope[(q * rope_stride + pos) * 4 + {0..3}] = (cos, sin) of the
 *                  head-dim pairs 2q and 2q + 1
 *   7 IMAGE        VAE predictor: scatter 20x20x3 patches into [frames, 3, 360, 640],
 *                  clamped to [-1, 1]
 *   8 GATED_RESID_LN as 4, then the next LayerNorm of the updated rows (ln_* fields)
 * K must be a multiple of 64 and N of 16. Split-K needs `workspace`. */
typedef struct OasisGemmArgs {
  const void* a; long long lda; /* bf16 */
  const void* w;                /* bf16 [N, K] */
  int m, n, k;
  int mode;
  void* out; long long ldo;
  const float* bias;
  const float* resid; long long ldr;
  const float* gate; long long ldg; int rows_per_frame;
  const float* rope; int rope_div; int rope_mod;
  int block_n; /* 0 = heuristic, else 32 / 64 / 128 / 256, or 512: 256 x 256 tiles on a 2-CTA pair */
  int splits;  /* 0 = heuristic, 1 = none */
  void* workspace; size_t workspace_bytes;
  int rope_dim; /* ROPE: width of the q (and k) section; 0 = 1024 (16 heads) */
  int rope_stride; /* ROPE: positions per row of the [16, positions, 4] table; 0 = rope_mod */
  /* GATED_RESID_LN (8): the LayerNorm + adaLN modulate of the new rows, written as
   * bf16 [M, 1024] to ln_out: (z - mean) rstd ln_mod[f ln_ld_mod + ln_scale_off + n]
   * + ln_mod[f ln_ld_mod + ln_shift_off + n], f = r / rows_per_frame (N = 1024). */
  void* ln_out; const float* ln_mod; long long ln_ld_mod, ln_shift_off, ln_scale_off; float ln_eps;
} OasisGemmArgs;

int oasis_gemm(const OasisGemmArgs* a, oasis_stream_t stream);
size_t oasis_gemm_workspace_size(int m, int n, int k);
/* The tile plan oasis_gemm would use for a call with a workspace and these
 * fields: tile width (512 = 256 x 256 tiles on a 2-CTA pair), K splits, whether
 * it runs on CTA pairs, and the split-K workspace bytes it needs. Any output
 * pointer may be NULL. Returns OASIS_ERR_INVALID_ARG for overrides oasis_gemm
 * would reject. No device work; usable without a GPU (148 SMs assumed). */
int oasis_gemm_plan(int m, int n, int k, int mode, int block_n, int splits, int* bn_out, int* splits_out,
                    int* pair_out, size_t* splitk_bytes_out);

/* oasis_gemm for callers that cannot allocate device memory (their allocator
 * belongs to a host framework, or allocation is not allowed where they run): the
 * split-K scratch comes from a library-owned fixed device array of
 * oasis_gemm_static_scratch_capacity() bytes (8 MiB, held on every GPU that loads
 * the library) instead of a->workspace, which is ignored. Problems needing more
 * scratch fail with OASIS_ERR_WORKSPACE. All calls share the array, so calls
 * that overlap on the GPU race; the first call on a device looks up the array's
 * address and should come before any stream capture. This entry point has no
 * counterpart in the reference. */
int oasis_gemm_static_scratch(const OasisGemmArgs* a, oasis_stream_t stream);
size_t oasis_gemm_static_scratch_capacity(void);

/* LayerNorm (eps, no affine) + adaLN modulate, or LayerNorm with affine w/b:
 * y_bf16[r] = LN(x[in_row]) * mul + add, where
 *   in_row = (r / P) * in_group + in_off + r % P
 *   modulated: frame = (r / P) * frame_mul + frame_add,
 *              add = mod[frame * ld_mod + shift_off + :], mul = mod[frame * ld_mod + scale_off + :]
 *   affine:    mul = affine_w, add = affine_b.
 * Replaces ttnn.layer_norm + ttnn.addcmul (oasis_inference.py:1053-1056) and
 * layernorm_d1024 (src/layernorm.py:15-96). Width is 1024. */
typedef struct OasisLayerNormArgs {
  const float* x; void* y; int rows_out;
  int P; long long in_group, in_off, frame_mul, frame_add;
  float eps;
  const float* mod; long long ld_mod, shift_off, scale_off;
  const float* affine_w; const float* affine_b;
} OasisLayerNormArgs;

int oasis_layernorm(const OasisLayerNormArgs* a, oasis_stream_t stream);

/* SiLU of fp32 x into bf16 y (silu_kernel, src/silu.py:8-47). n % 4 == 0. */
int oasis_silu_bf16(const float* x, void* y, long long n, oasis_stream_t stream);

/* Spatial / VAE attention: non-causal within groups of `seq` rows of a packed
 * qkv [rows, 3 heads 64] bf16 (q | k | v); out [rows, heads 64] bf16; heads is 16
 * for the full model, 16 / n on a rank of n-way tensor parallelism. Replaces
 * sdpa_spatial (src/sdpa.py:27-113, but over exactly `seq` keys) and the VAE ttnn SDPA. */
int oasis_attention_spatial(const void* qkv, void* out, int groups, int seq, int heads, oasis_stream_t stream);

/* Causal temporal attention per (session, patch, head) over T frames; token row
 * of (b, t, p) = (b T + t) 144 + p. Replaces sdpa_temporal_causal
 * (src/sdpa_causal.py:17-100) and its block-diagonal packing. */
/* The same full attention on the 5th-generation tensor cores (tcgen05.mma with
 * TMEM accumulators, TMA-fed): seq a multiple of 144. */
int oasis_attention_tc(const void* qkv, void* out, int groups, int seq, int heads, oasis_stream_t stream);
int oasis_attention_temporal(const void* qkv, void* out, int batch, int frames, int heads, oasis_stream_t stream);
/* The generated frame's query per (session, patch, head) against the cached
 * context keys/values plus its own: past_qkv [B, Tp, 144, 3 H 64], cur_qkv
 * [B, 144, 3 H 64], out [B, 144, H 64]. */
int oasis_attention_temporal_cached(const void* past_qkv, const void* cur_qkv, void* out, int batch, int past_frames,
                                    int heads, oasis_stream_t stream);

/* z[r, :1024] += gate[(r / rows_per_frame) ldg + :] * (x[r, :] + bias), gate NULL =
 * plain residual. Applies the bias, adaLN gate and residual after the all-reduce of a
 * row-parallel projection (tensor parallelism: `ttnn.all_reduce` then `ttnn.add` and
 * `ttnn.addcmul`, oasis_inference.py:1153-1165, 1191-1201). */
int oasis_gated_residual(float* z, const float* x, const float* bias, const float* gate, long long ldg,
                         int rows_per_frame, int rows, oasis_stream_t stream);

/* VAE post_quant_conv as a linear map: z[r] = latent[r, :16] . w + b. */
int oasis_post_quant(const float* latent, const float* w, const float* b, float* z, int rows,
                     oasis_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* OASIS_B200_H */
