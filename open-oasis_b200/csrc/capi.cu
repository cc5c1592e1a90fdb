// C ABI of the library (include/oasis_b200.h): argument checking, workspace
// carving, and the composite DiT / DDIM-step / VAE-decode drivers that issue the
// kernel sequence of one sub-block, one step and one decode on a caller stream.
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "../../include/oasis_b200.h"
#include "gemm.cuh"
#include "pointwise.cuh"
#include "status.h"

namespace oasis {

static thread_local char g_msg[512] = "";
static std::atomic<unsigned long long> g_launches{0};

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
  va_end(ap);
  return code;
}

int read_device_error(int reset);  // gemm.cu
int read_device_error_peer(int reset);  // peer.cu

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("OASIS_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

namespace {

constexpr int kD = 1024;
constexpr int kGemmRowBlock = 128;  // rows per GEMM tile: the LN-fused epilogue gives each CTA whole row blocks
constexpr int kP = 144;        // tokens per DiT frame
constexpr int kOut = 64;       // patch vector (2 x 2 x 16)
constexpr int kMlp = 4096;
constexpr int kVaeTok = 576;
constexpr float kScalingFactor = 0.07843137255f;

inline cudaStream_t S(oasis_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Bump allocator over a caller workspace (256-byte aligned slices).
struct Carve {
  uint8_t* base;
  size_t used = 0;
  size_t cap;
  Carve(void* b, size_t c) : base(static_cast<uint8_t*>(b)), cap(c) {}
  template <class T>
  T* take(size_t count) {
    used = (used + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + used) : nullptr;
    used += count * sizeof(T);
    return p;
  }
  bool ok() const { return used <= cap; }
};

size_t splitk_bytes_dit(int B, int T, bool last_only) {
  const int F = B * T, M = F * kP;
  size_t m = 0;
  auto upd = [&](size_t x) { m = x > m ? x : m; };
  upd(gemm_workspace_bytes(M, 3 * kD, kD));
  upd(gemm_workspace_bytes(M, kD, kD));
  upd(gemm_workspace_bytes(M, kMlp, kD));
  upd(gemm_workspace_bytes(M, kD, kMlp));
  upd(gemm_workspace_bytes(F, OASIS_ADALN_ROWS, kD));
  upd(gemm_workspace_bytes(last_only ? B * kP : M, kOut, kD));
  return m;
}

struct DitScratch {
  __nv_bfloat16* silu;
  float* adaln;
  __nv_bfloat16* xn;
  __nv_bfloat16* qkv;
  __nv_bfloat16* attn;
  __nv_bfloat16* h;
  void* splitk;
  size_t splitk_bytes;
};

size_t carve_dit(Carve& c, int B, int T, DitScratch* s, bool with_adaln = true) {
  const size_t F = (size_t)B * T, M = F * kP;
  DitScratch d;
  d.silu = with_adaln ? c.take<__nv_bfloat16>(F * kD) : nullptr;
  d.adaln = with_adaln ? c.take<float>(F * OASIS_ADALN_ROWS) : nullptr;
  d.xn = c.take<__nv_bfloat16>(M * kD);
  d.qkv = c.take<__nv_bfloat16>(M * 3 * kD);
  d.attn = c.take<__nv_bfloat16>(M * kD);
  d.h = c.take<__nv_bfloat16>(M * kMlp);
  d.splitk_bytes = splitk_bytes_dit(B, T, false);
  d.splitk = d.splitk_bytes ? c.take<uint8_t>(d.splitk_bytes) : nullptr;
  if (s) *s = d;
  return c.used;
}

GemmProblem gemm(const void* A, const void* W, int M, int N, int K, void* ws, size_t ws_bytes) {
  GemmProblem p;
  p.A = A;
  p.lda = K;
  p.W = W;
  p.M = M;
  p.N = N;
  p.K = K;
  p.workspace = ws;
  p.workspace_bytes = ws_bytes;
  return p;
}

// adaLN parameters of every sub-block and the final layer for `rows` frames:
// silu(cond) then ONE GEMM against the stacked adaLN weights.
int compute_adaln(const OasisDitWeights* w, const float* cond, int rows, __nv_bfloat16* silu, float* adaln,
                  void* splitk, size_t splitk_bytes, cudaStream_t st) {
  const long long ldm = (long long)w->num_subblocks * OASIS_ADALN_WIDTH + 2 * kD;
  OASIS_TRY(silu_bf16_launch(cond, silu, (long long)rows * kD, st));
  GemmProblem p = gemm(silu, w->adaln_w, rows, (int)ldm, kD, splitk, splitk_bytes);
  p.epi.mode = kEpiF32;
  p.epi.out = adaln;
  p.epi.ldo = ldm;
  p.epi.bias = w->adaln_b;
  return gemm_launch(p, st);
}

// Context caching across DDIM steps (oasis_inference.py:1218-1403): the context
// frames see only earlier frames (causal temporal attention) and keep the same
// conditioning at every step, so their rows are computed once per frame.
//   kSave: forward over the B x Tp context frames; each temporal sub-block's packed
//          QKV is written to its cache slot [B, Tp, 144, 3072] (the final layer is
//          skipped).
//   kUse:  forward over the generated frame only (T = 1 rows per session); at
//          temporal sub-blocks its query attends over the cached context keys
//          and values plus its own, at temporal position Tp.
enum KvMode { kKvNone = 0, kKvSave = 1, kKvUse = 2 };
struct KvCtx {
  int mode = kKvNone;
  __nv_bfloat16* cache = nullptr;  // [temporal sub-blocks][B, Tp, 144, 3072] bf16
  int past_frames = 0;             // Tp
};

size_t kv_slot_elems(int B, int Tp) { return (size_t)B * Tp * kP * 3 * kD; }

// The 32 sub-blocks and the final layer for B sessions x T frames, given the
// adaLN table [B T, ldm] of this step.
int dit_blocks(const OasisDitWeights* w, int B, int T, float* z, const float* adaln, float* v_out,
               int last_frame_only, const DitScratch& s, cudaStream_t st, const KvCtx& kv = KvCtx()) {
  const int F = B * T, M = F * kP;
  const int nsub = w->num_subblocks;
  const long long ldm = (long long)nsub * OASIS_ADALN_WIDTH + 2 * kD;
  float* const ad = const_cast<float*>(adaln);
  // OASIS_LN_FUSE=1 runs the next sub-block's first LayerNorm inside this
  // sub-block's FC2 epilogue (kEpiGatedResidLN; not after the last sub-block,
  // whose successor is the final layer's LN over other rows). Off by default:
  // measured at C4 it made the DiT step slower (76.1 vs 72.6 ms): the whole-row
  // scheduling and the serial LN pass cost more than the LayerNorm launch saves.
  static const bool fuse_ln = [] {
    const char* e = getenv("OASIS_LN_FUSE");
    return e && e[0] == '1';
  }();
  bool xn_ready = false;  // s.xn already holds this sub-block's first LayerNorm
  for (int i = 0; i < nsub; ++i) {
    const OasisDitSubBlock& sb = w->sub[i];
    const bool spatial = (i % 2) == 0;
    const long long off = (long long)i * OASIS_ADALN_WIDTH;
    LayerNormParams ln;
    ln.rows_out = M;
    ln.P = kP;
    ln.in_group = kP;
    ln.mod = ad;
    ln.ld_mod = ldm;
    ln.shift_off = off;
    ln.scale_off = off + kD;
    if (!xn_ready) OASIS_TRY(layernorm_launch(z, s.xn, ln, st));
    __nv_bfloat16* const slot =
        (!spatial && kv.mode != kKvNone) ? kv.cache + (size_t)(i / 2) * kv_slot_elems(B, kv.past_frames) : nullptr;
    __nv_bfloat16* const qkv = (!spatial && kv.mode == kKvSave) ? slot : s.qkv;
    {
      GemmProblem p = gemm(s.xn, sb.qkv_w, M, 3 * kD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiRopeBF16;
      p.epi.out = qkv;
      p.epi.ldo = 3 * kD;
      p.epi.rope = spatial ? w->rope_spatial : w->rope_temporal;
      p.epi.rope_div = spatial ? 1 : kP;
      p.epi.rope_mod = spatial ? kP : T;
      p.epi.rope_stride = spatial ? kP : OASIS_MAX_FRAMES;
      if (!spatial && kv.mode == kKvUse) {  // every row sits at temporal position Tp
        p.epi.rope = w->rope_temporal + (size_t)kv.past_frames * 4;
        p.epi.rope_div = 1;
        p.epi.rope_mod = 1;
      }
      OASIS_TRY(gemm_launch(p, st));
    }
    if (spatial)
      OASIS_TRY(attention_full_launch(qkv, s.attn, F, kP, 16, st));
    else if (kv.mode == kKvUse)
      OASIS_TRY(attention_temporal_cached_launch(slot, qkv, s.attn, B, kv.past_frames, kP, 16, st));
    else
      OASIS_TRY(attention_temporal_launch(qkv, s.attn, B, T, kP, 16, st));
    {
      GemmProblem p = gemm(s.attn, sb.out_w, M, kD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiGatedResid;
      p.epi.out = z;
      p.epi.ldo = kD;
      p.epi.resid = z;
      p.epi.ldr = kD;
      p.epi.bias = sb.out_b;
      p.epi.gate = ad + off + 2 * kD;
      p.epi.ldg = ldm;
      p.epi.rows_per_frame = kP;
      OASIS_TRY(gemm_launch(p, st));
    }
    ln.shift_off = off + 3 * kD;
    ln.scale_off = off + 4 * kD;
    OASIS_TRY(layernorm_launch(z, s.xn, ln, st));
    {
      GemmProblem p = gemm(s.xn, sb.fc1_w, M, kMlp, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiGeluTanhBF16;
      p.epi.out = s.h;
      p.epi.ldo = kMlp;
      p.epi.bias = sb.fc1_b;
      OASIS_TRY(gemm_launch(p, st));
    }
    {
      GemmProblem p = gemm(s.h, sb.fc2_w, M, kD, kMlp, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiGatedResid;
      p.epi.out = z;
      p.epi.ldo = kD;
      p.epi.resid = z;
      p.epi.ldr = kD;
      p.epi.bias = sb.fc2_b;
      p.epi.gate = ad + off + 5 * kD;
      p.epi.ldg = ldm;
      p.epi.rows_per_frame = kP;
      // whole-row blocks need at least one per SM to keep every SM busy
      xn_ready = fuse_ln && i + 1 < nsub && M >= num_sms() * kGemmRowBlock;
      if (xn_ready) {
        p.epi.mode = kEpiGatedResidLN;
        p.ln.out = s.xn;
        p.ln.mod = ad;
        p.ln.ld_mod = ldm;
        p.ln.shift_off = off + OASIS_ADALN_WIDTH;  // sub-block i + 1: (shift, 1 + scale) of its attention LN
        p.ln.scale_off = off + OASIS_ADALN_WIDTH + kD;
        p.ln.eps = 1e-6f;
      }
      OASIS_TRY(gemm_launch(p, st));
    }
  }

  if (kv.mode == kKvSave) return OASIS_OK;  // only the cache is wanted
  // Final layer: LN + final adaLN modulate (only the rows that are returned) + linear.
  const long long foff = (long long)nsub * OASIS_ADALN_WIDTH;
  LayerNormParams ln;
  ln.P = kP;
  ln.mod = ad;
  ln.ld_mod = ldm;
  ln.shift_off = foff;
  ln.scale_off = foff + kD;
  if (last_frame_only) {
    ln.rows_out = B * kP;
    ln.in_group = (long long)T * kP;
    ln.in_off = (long long)(T - 1) * kP;
    ln.frame_mul = T;
    ln.frame_add = T - 1;
  } else {
    ln.rows_out = M;
    ln.in_group = kP;
  }
  OASIS_TRY(layernorm_launch(z, s.xn, ln, st));
  GemmProblem p = gemm(s.xn, w->final_w, ln.rows_out, kOut, kD, s.splitk, s.splitk_bytes);
  p.epi.mode = kEpiF32;
  p.epi.out = v_out;
  p.epi.ldo = kOut;
  p.epi.bias = w->final_b;
  return gemm_launch(p, st);
}

int dit_forward_impl(const OasisDitWeights* w, const OasisDitArgs* a, cudaStream_t st) {
  OASIS_REQUIRE(w && a, "dit_forward: null argument");
  const int B = a->batch, T = a->frames;
  OASIS_REQUIRE(B > 0 && T > 0 && T <= 32, "dit_forward: batch=%d frames=%d (need frames in [1, 32])", B, T);
  OASIS_REQUIRE(a->z && a->cond && a->v_out, "dit_forward: null tensor");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "dit_forward: num_subblocks=%d",
                w->num_subblocks);
  Carve c(a->workspace, a->workspace_bytes);
  DitScratch s;
  carve_dit(c, B, T, &s);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "dit_forward: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  OASIS_TRY(compute_adaln(w, a->cond, B * T, s.silu, s.adaln, s.splitk, s.splitk_bytes, st));
  return dit_blocks(w, B, T, a->z, s.adaln, a->v_out, a->last_frame_only, s, st);
}

size_t step_ws(int B, int T, DitScratch* s, float** z, float** v, void* base, size_t cap) {
  Carve c(base, cap);
  carve_dit(c, B, T, s);
  float* zz = c.take<float>((size_t)B * T * kP * kD);
  float* vv = c.take<float>((size_t)B * kP * kOut);
  if (z) *z = zz;
  if (v) *v = vv;
  return c.used;
}

struct VaeScratch {
  float* z;
  __nv_bfloat16* xn;
  __nv_bfloat16* qkv;
  __nv_bfloat16* attn;
  __nv_bfloat16* h;
  void* splitk;
  size_t splitk_bytes;
};

size_t carve_vae(Carve& c, int B, VaeScratch* s) {
  const size_t R = (size_t)B * kVaeTok;
  VaeScratch d;
  d.z = c.take<float>(R * kD);
  d.xn = c.take<__nv_bfloat16>(R * kD);
  d.qkv = c.take<__nv_bfloat16>(R * 3 * kD);
  d.attn = c.take<__nv_bfloat16>(R * kD);
  d.h = c.take<__nv_bfloat16>(R * kMlp);
  size_t m = 0;
  auto upd = [&](size_t x) { m = x > m ? x : m; };
  upd(gemm_workspace_bytes((int)R, 3 * kD, kD));
  upd(gemm_workspace_bytes((int)R, kD, kD));
  upd(gemm_workspace_bytes((int)R, kMlp, kD));
  upd(gemm_workspace_bytes((int)R, kD, kMlp));
  upd(gemm_workspace_bytes((int)R, 1200, kD));
  d.splitk_bytes = m;
  d.splitk = m ? c.take<uint8_t>(m) : nullptr;
  if (s) *s = d;
  return c.used;
}

// num_blocks pre-LN ViT blocks over the residual stream s.z [B * 576, 1024]
// (decoder: oasis_inference.py:1546-1618; the encoder has the same blocks), then the
// final LayerNorm (norm_w, norm_b) into s.xn as the next GEMM's operand.
int vae_block_stack(const OasisVaeBlock* blk, int nb, const float* rope, const float* norm_w, const float* norm_b,
                    int R, const VaeScratch& s, cudaStream_t st) {
  LayerNormParams ln;
  ln.rows_out = R;
  ln.P = R;
  ln.in_group = R;
  const int B = R / kVaeTok;
  for (int i = 0; i < nb; ++i) {
    const OasisVaeBlock& b = blk[i];
    ln.affine_w = b.norm1_w;
    ln.affine_b = b.norm1_b;
    OASIS_TRY(layernorm_launch(s.z, s.xn, ln, st));
    {
      GemmProblem p = gemm(s.xn, b.qkv_w, R, 3 * kD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiRopeBF16;
      p.epi.out = s.qkv;
      p.epi.ldo = 3 * kD;
      p.epi.bias = b.qkv_b;
      p.epi.rope = rope;
      p.epi.rope_div = 1;
      p.epi.rope_mod = kVaeTok;
      p.epi.rope_stride = kVaeTok;
      OASIS_TRY(gemm_launch(p, st));
    }
    OASIS_TRY(attention_full_launch(s.qkv, s.attn, B, kVaeTok, 16, st));
    {
      GemmProblem p = gemm(s.attn, b.proj_w, R, kD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiResid;
      p.epi.out = s.z;
      p.epi.ldo = kD;
      p.epi.resid = s.z;
      p.epi.ldr = kD;
      p.epi.bias = b.proj_b;
      OASIS_TRY(gemm_launch(p, st));
    }
    ln.affine_w = b.norm2_w;
    ln.affine_b = b.norm2_b;
    OASIS_TRY(layernorm_launch(s.z, s.xn, ln, st));
    {
      GemmProblem p = gemm(s.xn, b.fc1_w, R, kMlp, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiGeluErfBF16;
      p.epi.out = s.h;
      p.epi.ldo = kMlp;
      p.epi.bias = b.fc1_b;
      OASIS_TRY(gemm_launch(p, st));
    }
    {
      GemmProblem p = gemm(s.h, b.fc2_w, R, kD, kMlp, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiResid;
      p.epi.out = s.z;
      p.epi.ldo = kD;
      p.epi.resid = s.z;
      p.epi.ldr = kD;
      p.epi.bias = b.fc2_b;
      OASIS_TRY(gemm_launch(p, st));
    }
  }
  ln.affine_w = norm_w;
  ln.affine_b = norm_b;
  return layernorm_launch(s.z, s.xn, ln, st);
}

int vae_decode_impl(const OasisVaeWeights* w, const OasisVaeArgs* a, cudaStream_t st) {
  OASIS_REQUIRE(w && a, "vae_decode: null argument");
  const int B = a->batch;
  OASIS_REQUIRE(B > 0, "vae_decode: batch=%d", B);
  OASIS_REQUIRE(a->latent && a->image, "vae_decode: null tensor");
  Carve c(a->workspace, a->workspace_bytes);
  VaeScratch s;
  carve_vae(c, B, &s);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "vae_decode: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  const int R = B * kVaeTok;
  OASIS_TRY(post_quant_launch(a->latent, w->post_quant_w, w->post_quant_b, s.z, R, st));
  OASIS_REQUIRE(w->num_blocks >= 0 && w->num_blocks <= OASIS_VAE_BLOCKS, "vae_decode: num_blocks=%d", w->num_blocks);
  OASIS_TRY(vae_block_stack(w->blk, w->num_blocks, w->rope, w->norm_w, w->norm_b, R, s, st));
  GemmProblem p = gemm(s.xn, w->pred_w, R, 1200, kD, s.splitk, s.splitk_bytes);
  p.epi.mode = kEpiImage;
  p.epi.out = a->image;
  p.epi.bias = w->pred_b;
  p.epi.img_grid_w = 32;
  p.epi.img_tokens = kVaeTok;
  p.epi.img_patch = 20;
  return gemm_launch(p, st);
}


// VAE encoder scratch: the decoder's (the blocks are the same) plus the patch rows
// [B * 576, OASIS_VAE_ENC_K] bf16 and the moments [B * 576, 32] fp32.
size_t carve_vae_enc(Carve& c, int B, VaeScratch* s, __nv_bfloat16** patches, float** moments) {
  VaeScratch d;
  carve_vae(c, B, &d);
  const size_t R = (size_t)B * kVaeTok;
  __nv_bfloat16* p = c.take<__nv_bfloat16>(R * OASIS_VAE_ENC_K);
  float* m = c.take<float>(R * 32);
  // the split-K area must also cover the encoder's own GEMMs (patch embed, quant)
  size_t need = gemm_workspace_bytes((int)R, kD, OASIS_VAE_ENC_K);
  const size_t q = gemm_workspace_bytes((int)R, 32, kD);
  need = q > need ? q : need;
  if (need > d.splitk_bytes) {
    d.splitk = c.take<uint8_t>(need);
    d.splitk_bytes = need;
  }
  if (s) *s = d;
  if (patches) *patches = p;
  if (moments) *moments = m;
  return c.used;
}

int vae_encode_impl(const OasisVaeEncoderWeights* w, const OasisVaeEncodeArgs* a, cudaStream_t st) {
  OASIS_REQUIRE(w && a, "vae_encode: null argument");
  const int B = a->batch;
  OASIS_REQUIRE(B > 0, "vae_encode: batch=%d", B);
  OASIS_REQUIRE(a->image && (a->latent || a->chunk), "vae_encode: null image, or neither latent nor chunk");
  OASIS_REQUIRE(w->num_blocks >= 0 && w->num_blocks <= OASIS_VAE_BLOCKS, "vae_encode: num_blocks=%d", w->num_blocks);
  OASIS_REQUIRE(w->patch_w && w->quant_w && w->norm_w && w->norm_b && (w->num_blocks == 0 || w->rope),
                "vae_encode: null weight");
  Carve c(a->workspace, a->workspace_bytes);
  VaeScratch s;
  __nv_bfloat16* patches;
  float* moments;
  carve_vae_enc(c, B, &s, &patches, &moments);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "vae_encode: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  const int R = B * kVaeTok;
  OASIS_TRY(image_patchify_launch(a->image, patches, B, OASIS_VAE_ENC_K, st));
  {
    GemmProblem p = gemm(patches, w->patch_w, R, kD, OASIS_VAE_ENC_K, s.splitk, s.splitk_bytes);
    p.epi.mode = kEpiF32;
    p.epi.out = s.z;
    p.epi.ldo = kD;
    p.epi.bias = w->patch_b;
    OASIS_TRY(gemm_launch(p, st));
  }
  OASIS_TRY(vae_block_stack(w->blk, w->num_blocks, w->rope, w->norm_w, w->norm_b, R, s, st));
  {
    GemmProblem p = gemm(s.xn, w->quant_w, R, 32, kD, s.splitk, s.splitk_bytes);
    p.epi.mode = kEpiF32;
    p.block_n = 32;  // one tile spans the 32 moments
    p.epi.out = moments;
    p.epi.ldo = 32;
    p.epi.bias = w->quant_b;
    OASIS_TRY(gemm_launch(p, st));
  }
  return moments_to_latent_launch(moments, a->latent, a->chunk, B, kScalingFactor, st);
}

constexpr int kMaxFrameSteps = 64;

struct FrameScratch {
  __nv_bfloat16* silu;  // [steps B T, 1024]
  float* adaln;         // [steps B T, 6144 S + 2048]
  float* z;             // [B T 144, 1024]
  float* v;             // [B 144, 64]
  float* latent;        // [B, 576, 16]
  void* shared;         // DiT step scratch, later reused by the VAE decode
  size_t shared_bytes;
};

size_t carve_frame(Carve& c, int B, int T, int S, FrameScratch* f) {
  const size_t F = (size_t)B * T;
  FrameScratch d;
  d.silu = c.take<__nv_bfloat16>((size_t)S * F * kD);
  d.adaln = c.take<float>((size_t)S * F * OASIS_ADALN_ROWS);
  d.z = c.take<float>(F * kP * kD);
  d.v = c.take<float>((size_t)B * kP * kOut);
  d.latent = c.take<float>((size_t)B * kVaeTok * 16);
  Carve dit(nullptr, 0), vae(nullptr, 0);
  carve_dit(dit, B, T, nullptr, false);
  carve_vae(vae, B, nullptr);
  d.shared_bytes = (dit.used > vae.used ? dit.used : vae.used) + 256;
  d.shared = c.take<uint8_t>(d.shared_bytes);
  if (f) *f = d;
  return c.used;
}

int generate_frame_impl(const OasisDitWeights* w, const OasisVaeWeights* vw, const OasisFrameArgs* a,
                        cudaStream_t st) {
  OASIS_REQUIRE(w && a, "generate_frame: null argument");
  const int B = a->batch, T = a->frames, S = a->steps;
  OASIS_REQUIRE(B > 0 && T > 0 && T <= 32, "generate_frame: batch=%d frames=%d", B, T);
  OASIS_REQUIRE(S > 0 && S <= kMaxFrameSteps, "generate_frame: steps=%d outside [1, %d]", S, kMaxFrameSteps);
  OASIS_REQUIRE(a->chunk && a->cond && a->coeffs, "generate_frame: null tensor");
  OASIS_REQUIRE(T == 1 || a->context_z, "generate_frame: frames > 1 needs context_z");
  OASIS_REQUIRE(a->skip_decode || (vw && a->image), "generate_frame: decoding needs VAE weights and an image");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "generate_frame: num_subblocks");
  Carve c(a->workspace, a->workspace_bytes);
  FrameScratch f;
  carve_frame(c, B, T, S, &f);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "generate_frame: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  Carve dc(f.shared, f.shared_bytes);
  DitScratch s;
  carve_dit(dc, B, T, &s, false);
  const int F = B * T;
  const long long ldm = (long long)w->num_subblocks * OASIS_ADALN_WIDTH + 2 * kD;
  // adaLN tables of all steps at once: the stacked weights stream from HBM once per frame.
  OASIS_TRY(compute_adaln(w, a->cond, S * F, f.silu, f.adaln, s.splitk, s.splitk_bytes, st));
  for (int i = 0; i < S; ++i) {
    if (T > 1) {
      const size_t ctx_bytes = (size_t)(T - 1) * kP * kD * sizeof(float);
      cudaError_t e = cudaMemcpy2DAsync(f.z, (size_t)T * kP * kD * sizeof(float), a->context_z, ctx_bytes,
                                        ctx_bytes, B, cudaMemcpyDeviceToDevice, st);
      if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "generate_frame: context copy: %s", cudaGetErrorString(e));
    }
    PatchEmbedParams pe;
    pe.rows = B * kP;
    pe.P = kP;
    pe.out_group = (long long)T * kP;
    pe.out_off = (long long)(T - 1) * kP;
    OASIS_TRY(patch_embed_launch(a->chunk, w->embed_w, w->embed_b, f.z, pe, st));
    OASIS_TRY(dit_blocks(w, B, T, f.z, f.adaln + (size_t)i * F * ldm, f.v, 1, s, st));
    const OasisDdimCoeffs& k = a->coeffs[i];
    DdimCoeffs dk{k.at_sqrt, k.one_minus_at_sqrt, k.inv_at_sqrt, k.inv_sigma, k.an_sqrt, k.one_minus_an_sqrt};
    OASIS_TRY(ddim_launch(a->chunk, f.v, dk, (long long)B * kP * kOut, st));
  }
  if (a->skip_decode) return OASIS_OK;
  OASIS_TRY(bridge_launch(a->chunk, f.latent, B, 1.0f / kScalingFactor, st));
  OasisVaeArgs va{B, f.latent, a->image, f.shared, f.shared_bytes};
  return vae_decode_impl(vw, &va, st);
}

// ---- tensor parallelism ----

struct TpScratch {
  __nv_bfloat16* silu;
  float* adaln;
  __nv_bfloat16* xn;
  __nv_bfloat16* qkv;   // [M, 3 HD]
  __nv_bfloat16* attn;  // [M, HD]
  __nv_bfloat16* h;     // [M, 4 HD]
  void* splitk;
  size_t splitk_bytes;
};

size_t carve_tp(Carve& c, int B, int T, int heads, TpScratch* s) {
  const size_t F = (size_t)B * T, M = F * kP, HD = (size_t)heads * 64;
  TpScratch d;
  d.silu = c.take<__nv_bfloat16>(F * kD);
  d.adaln = c.take<float>(F * OASIS_ADALN_ROWS);
  d.xn = c.take<__nv_bfloat16>(M * kD);
  d.qkv = c.take<__nv_bfloat16>(M * 3 * HD);
  d.attn = c.take<__nv_bfloat16>(M * HD);
  d.h = c.take<__nv_bfloat16>(M * 4 * HD);
  size_t m = 0;
  auto upd = [&](size_t x) { m = x > m ? x : m; };
  upd(gemm_workspace_bytes((int)M, (int)(3 * HD), kD));
  upd(gemm_workspace_bytes((int)M, kD, (int)HD));
  upd(gemm_workspace_bytes((int)M, (int)(4 * HD), kD));
  upd(gemm_workspace_bytes((int)M, kD, (int)(4 * HD)));
  upd(gemm_workspace_bytes((int)F, OASIS_ADALN_ROWS, kD));
  upd(gemm_workspace_bytes(B * kP, kOut, kD));
  d.splitk_bytes = m;
  d.splitk = m ? c.take<uint8_t>(m) : nullptr;
  if (s) *s = d;
  return c.used;
}

int tp_forward_impl(const OasisDitWeights* w, const OasisTpArgs* a, cudaStream_t st) {
  OASIS_REQUIRE(w && a, "dit_forward_tp: null argument");
  const int B = a->batch, T = a->frames, H = a->heads;
  OASIS_REQUIRE(B > 0 && T > 0 && T <= OASIS_MAX_FRAMES, "dit_forward_tp: batch=%d frames=%d", B, T);
  OASIS_REQUIRE(H >= 1 && H <= 16 && 16 % H == 0, "dit_forward_tp: heads=%d must divide 16", H);
  OASIS_REQUIRE(a->z && a->cond && a->v_out && a->partial && a->allreduce, "dit_forward_tp: null tensor or collective");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "dit_forward_tp: num_subblocks");
  Carve c(a->workspace, a->workspace_bytes);
  TpScratch s;
  carve_tp(c, B, T, H, &s);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "dit_forward_tp: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  const int F = B * T, M = F * kP, HD = H * 64;
  const long long ldm = (long long)w->num_subblocks * OASIS_ADALN_WIDTH + 2 * kD;
  OASIS_TRY(compute_adaln(w, a->cond, F, s.silu, s.adaln, s.splitk, s.splitk_bytes, st));
  float* z = a->z;
  auto reduce = [&](const char* what) -> int {
    const int rc = a->allreduce(a->partial, (size_t)M * kD, a->allreduce_user, st);
    if (rc != 0) return set_error(rc < 0 ? rc : OASIS_ERR_CUDA, "dit_forward_tp: allreduce after %s returned %d", what, rc);
    return OASIS_OK;
  };
  for (int i = 0; i < w->num_subblocks; ++i) {
    const OasisDitSubBlock& sb = w->sub[i];
    const bool spatial = (i % 2) == 0;
    const long long off = (long long)i * OASIS_ADALN_WIDTH;
    LayerNormParams ln;
    ln.rows_out = M;
    ln.P = kP;
    ln.in_group = kP;
    ln.mod = s.adaln;
    ln.ld_mod = ldm;
    ln.shift_off = off;
    ln.scale_off = off + kD;
    OASIS_TRY(layernorm_launch(z, s.xn, ln, st));
    {
      GemmProblem p = gemm(s.xn, sb.qkv_w, M, 3 * HD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiRopeBF16;
      p.epi.out = s.qkv;
      p.epi.ldo = 3 * HD;
      p.epi.rope = spatial ? w->rope_spatial : w->rope_temporal;
      p.epi.rope_div = spatial ? 1 : kP;
      p.epi.rope_mod = spatial ? kP : T;
      p.epi.rope_stride = spatial ? kP : OASIS_MAX_FRAMES;
      p.epi.rope_dim = HD;
      OASIS_TRY(gemm_launch(p, st));
    }
    if (spatial)
      OASIS_TRY(attention_full_launch(s.qkv, s.attn, F, kP, H, st));
    else
      OASIS_TRY(attention_temporal_launch(s.qkv, s.attn, B, T, kP, H, st));
    {
      GemmProblem p = gemm(s.attn, sb.out_w, M, kD, HD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiF32;
      p.epi.out = a->partial;
      p.epi.ldo = kD;
      OASIS_TRY(gemm_launch(p, st));
    }
    OASIS_TRY(reduce("O"));
    OASIS_TRY(gated_residual_launch(z, a->partial, sb.out_b, s.adaln + off + 2 * kD, ldm, kP, M, st));
    ln.shift_off = off + 3 * kD;
    ln.scale_off = off + 4 * kD;
    OASIS_TRY(layernorm_launch(z, s.xn, ln, st));
    {
      GemmProblem p = gemm(s.xn, sb.fc1_w, M, 4 * HD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiGeluTanhBF16;
      p.epi.out = s.h;
      p.epi.ldo = 4 * HD;
      p.epi.bias = sb.fc1_b;
      OASIS_TRY(gemm_launch(p, st));
    }
    {
      GemmProblem p = gemm(s.h, sb.fc2_w, M, kD, 4 * HD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiF32;
      p.epi.out = a->partial;
      p.epi.ldo = kD;
      OASIS_TRY(gemm_launch(p, st));
    }
    OASIS_TRY(reduce("FC2"));
    OASIS_TRY(gated_residual_launch(z, a->partial, sb.fc2_b, s.adaln + off + 5 * kD, ldm, kP, M, st));
  }
  const long long foff = (long long)w->num_subblocks * OASIS_ADALN_WIDTH;
  LayerNormParams ln;
  ln.P = kP;
  ln.mod = s.adaln;
  ln.ld_mod = ldm;
  ln.shift_off = foff;
  ln.scale_off = foff + kD;
  ln.rows_out = B * kP;
  ln.in_group = (long long)T * kP;
  ln.in_off = (long long)(T - 1) * kP;
  ln.frame_mul = T;
  ln.frame_add = T - 1;
  OASIS_TRY(layernorm_launch(z, s.xn, ln, st));
  GemmProblem p = gemm(s.xn, w->final_w, B * kP, kOut, kD, s.splitk, s.splitk_bytes);
  p.epi.mode = kEpiF32;
  p.epi.out = a->v_out;
  p.epi.ldo = kOut;
  p.epi.bias = w->final_b;
  return gemm_launch(p, st);
}

// ---- sequence-parallel tensor parallelism ----
// Per-rank scratch: the adaLN table of the owned frames, the local heads' QKV,
// attention output and MLP hidden over all rows, split-K partials. The
// communication buffers are the caller's (OasisTpSpArgs).
struct TpSpScratch {
  __nv_bfloat16* silu;
  float* adaln;
  __nv_bfloat16* qkv;
  __nv_bfloat16* attn;
  __nv_bfloat16* h;
  void* splitk;
  size_t splitk_bytes;
};

size_t carve_tp_sp(Carve& c, int B, int T, int heads, int world, TpSpScratch* s) {
  const size_t Fl = (size_t)(B / world) * T, M = (size_t)B * T * kP, HD = (size_t)heads * 64;
  TpSpScratch d;
  d.silu = c.take<__nv_bfloat16>(Fl * kD);
  d.adaln = c.take<float>(Fl * OASIS_ADALN_ROWS);
  d.qkv = c.take<__nv_bfloat16>(M * 3 * HD);
  d.attn = c.take<__nv_bfloat16>(M * HD);
  d.h = c.take<__nv_bfloat16>(M * 4 * HD);
  size_t m = 0;
  auto upd = [&](size_t x) { m = x > m ? x : m; };
  upd(gemm_workspace_bytes((int)M, (int)(3 * HD), kD));
  upd(gemm_workspace_bytes((int)M, kD, (int)HD));
  upd(gemm_workspace_bytes((int)M, (int)(4 * HD), kD));
  upd(gemm_workspace_bytes((int)M, kD, (int)(4 * HD)));
  upd(gemm_workspace_bytes((int)Fl, OASIS_ADALN_ROWS, kD));
  upd(gemm_workspace_bytes((B / world) * kP, kOut, kD));
  d.splitk_bytes = m;
  d.splitk = m ? c.take<uint8_t>(m) : nullptr;
  if (s) *s = d;
  return c.used;
}

// Stream handoff events of the overlapped sequence-parallel forward, created on
// first use per device (events hold no device memory). Slot 0 orders compute ->
// communication (recorded and waited at once, so one event serves); slots
// 1 + k mark the completion of chunk k's latest collective. A wait takes the
// event's state at the time it is enqueued, so every slot is reused.
constexpr int kTpMaxChunks = 8;
cudaEvent_t handoff_event(int slot) {
  static std::mutex mu;
  static cudaEvent_t ev[64][1 + kTpMaxChunks] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(mu);
  cudaEvent_t& e = ev[dev & 63][slot];
  if (!e && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) e = nullptr;
  return e;
}

int tp_sp_forward_impl(const OasisDitWeights* w, const OasisTpSpArgs* a, cudaStream_t st) {
  OASIS_REQUIRE(w && a, "dit_forward_tp_sp: null argument");
  const int B = a->batch, T = a->frames, H = a->heads, n = a->world, rk = a->rank;
  OASIS_REQUIRE(n >= 1 && rk >= 0 && rk < n && H * n == 16, "dit_forward_tp_sp: rank %d of %d with %d heads", rk, n, H);
  OASIS_REQUIRE(B > 0 && B % n == 0 && T > 0 && T <= OASIS_MAX_FRAMES,
                "dit_forward_tp_sp: batch=%d (a multiple of world=%d) frames=%d", B, n, T);
  OASIS_REQUIRE(a->partial_dtype == OASIS_DTYPE_F32 || a->partial_dtype == OASIS_DTYPE_BF16,
                "dit_forward_tp_sp: partial_dtype=%d", a->partial_dtype);
  OASIS_REQUIRE(a->z && a->cond && a->v_out && a->partial && a->shard && a->xn_local && a->xn && a->v_local,
                "dit_forward_tp_sp: null tensor");
  OASIS_REQUIRE(a->reduce_scatter && a->all_gather, "dit_forward_tp_sp: null collective");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "dit_forward_tp_sp: num_subblocks");
  const int Bl = B / n;
  const int C = a->chunks > 1 ? a->chunks : 1;
  OASIS_REQUIRE(Bl % C == 0 && C <= kTpMaxChunks, "dit_forward_tp_sp: chunks=%d must divide the %d sessions per rank "
                "(at most %d)", C, Bl, kTpMaxChunks);
  Carve c(a->workspace, a->workspace_bytes);
  TpSpScratch s;
  carve_tp_sp(c, B, T, H, n, &s);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "dit_forward_tp_sp: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  const int Fl = Bl * T, Ml = Fl * kP, HD = H * 64;
  const int Bc = Bl / C, Mc = Bc * T * kP;  // one chunk: Bc sessions of this rank, Mc rows
  const int Bg = Bc * n, Mg = Mc * n;       // the chunk gathered over the ranks
  const bool bf16_part = a->partial_dtype == OASIS_DTYPE_BF16;
  const size_t pe = bf16_part ? 2 : 4;
  const long long ldm = (long long)w->num_subblocks * OASIS_ADALN_WIDTH + 2 * kD;
  // Compute on `st`; with a communication stream the collectives go there and the
  // two streams hand chunks over with events, so the collective of chunk k
  // overlaps the compute of chunk k + 1.
  cudaStream_t cs = a->comm_stream ? reinterpret_cast<cudaStream_t>(a->comm_stream) : st;
  const bool two = cs != st;
  cudaEvent_t ev[1 + kTpMaxChunks] = {};
  if (two) {
    for (int k = 0; k <= C; ++k)
      if (!(ev[k] = handoff_event(k))) return set_error(OASIS_ERR_CUDA, "dit_forward_tp_sp: cudaEventCreate failed");
  }
  auto to_comm = [&]() -> int {  // the collective about to be issued sees everything computed so far
    if (!two) return OASIS_OK;
    if (cudaEventRecord(ev[0], st) != cudaSuccess || cudaStreamWaitEvent(cs, ev[0], 0) != cudaSuccess)
      return set_error(OASIS_ERR_CUDA, "dit_forward_tp_sp: stream handoff failed");
    return OASIS_OK;
  };
  auto mark = [&](int k) -> int {  // chunk k's collective is issued: remember where it ends
    if (!two) return OASIS_OK;
    if (cudaEventRecord(ev[1 + k], cs) != cudaSuccess) return set_error(OASIS_ERR_CUDA, "dit_forward_tp_sp: event");
    return OASIS_OK;
  };
  auto await = [&](int k) -> int {  // compute on chunk k waits for its collective
    if (!two) return OASIS_OK;
    if (cudaStreamWaitEvent(st, ev[1 + k], 0) != cudaSuccess)
      return set_error(OASIS_ERR_CUDA, "dit_forward_tp_sp: stream handoff failed");
    return OASIS_OK;
  };
  // With overlap, the persistent kernels leave `reserve_sms` SMs to the collectives
  // (restored when this call returns, on every path).
  struct Reserve {
    explicit Reserve(int n) { set_sm_reserve(n); }
    ~Reserve() { set_sm_reserve(0); }
  } reserve(two ? a->reserve_sms : 0);
  OASIS_TRY(compute_adaln(w, a->cond, Fl, s.silu, s.adaln, s.splitk, s.splitk_bytes, st));
  float* z = a->z;
  auto xn_loc = static_cast<__nv_bfloat16*>(a->xn_local);
  auto xn = static_cast<__nv_bfloat16*>(a->xn);
  auto part = static_cast<uint8_t*>(a->partial);
  auto shard = static_cast<uint8_t*>(a->shard);
  auto collective = [&](oasis_collective_fn fn, const void* send, void* recv, size_t count, int dtype,
                        const char* what) -> int {
    const int rc = fn(send, recv, count, dtype, a->user, cs);
    if (rc != 0) return set_error(rc < 0 ? rc : OASIS_ERR_CUDA, "dit_forward_tp_sp: %s returned %d", what, rc);
    return OASIS_OK;
  };
  // chunk k: owned rows [k Mc, (k + 1) Mc); its gathered rows [k Mg, (k + 1) Mg) of xn / partial
  auto ln_chunk = [&](int k, long long shift, long long scale) -> int {
    LayerNormParams ln;
    ln.rows_out = Mc;
    ln.P = kP;
    ln.in_group = kP;
    ln.mod = s.adaln + (size_t)k * Bc * T * ldm;
    ln.ld_mod = ldm;
    ln.shift_off = shift;
    ln.scale_off = scale;
    return layernorm_launch(z + (size_t)k * Mc * kD, xn_loc + (size_t)k * Mc * kD, ln, st);
  };
  auto gather_chunks = [&](long long shift, long long scale, const char* what) -> int {
    for (int k = 0; k < C; ++k) {
      OASIS_TRY(ln_chunk(k, shift, scale));
      OASIS_TRY(to_comm());
      OASIS_TRY(collective(a->all_gather, xn_loc + (size_t)k * Mc * kD, xn + (size_t)k * Mg * kD, (size_t)Mc * kD,
                           OASIS_DTYPE_BF16, what));
      OASIS_TRY(mark(k));
    }
    return OASIS_OK;
  };
  // row-parallel projection of chunk k into its partial rows, then their reduce-scatter
  auto project_scatter = [&](int k, const __nv_bfloat16* in, const void* wt, int K, const char* what) -> int {
    GemmProblem p = gemm(in, wt, Mg, kD, K, s.splitk, s.splitk_bytes);
    p.epi.mode = bf16_part ? kEpiBF16 : kEpiF32;
    p.epi.out = part + (size_t)k * Mg * kD * pe;
    p.epi.ldo = kD;
    OASIS_TRY(gemm_launch(p, st));
    OASIS_TRY(to_comm());
    OASIS_TRY(collective(a->reduce_scatter, part + (size_t)k * Mg * kD * pe, shard + (size_t)k * Mc * kD * pe,
                         (size_t)Mc * kD, a->partial_dtype, what));
    return mark(k);
  };
  auto residual_chunk = [&](int k, const float* bias, long long gate_off) -> int {
    const float* gate = s.adaln + (size_t)k * Bc * T * ldm + gate_off;
    float* zk = z + (size_t)k * Mc * kD;
    if (bf16_part)
      return gated_residual_bf16_launch(zk, reinterpret_cast<const __nv_bfloat16*>(shard + (size_t)k * Mc * kD * pe),
                                        bias, gate, ldm, kP, Mc, st);
    return gated_residual_launch(zk, reinterpret_cast<const float*>(shard + (size_t)k * Mc * kD * pe), bias, gate,
                                 ldm, kP, Mc, st);
  };
  for (int i = 0; i < w->num_subblocks; ++i) {
    const OasisDitSubBlock& sb = w->sub[i];
    const bool spatial = (i % 2) == 0;
    const long long off = (long long)i * OASIS_ADALN_WIDTH;
    OASIS_TRY(gather_chunks(off, off + kD, "all_gather before QKV"));
    for (int k = 0; k < C; ++k) {
      OASIS_TRY(await(k));  // chunk k's xn has landed
      const __nv_bfloat16* xk = xn + (size_t)k * Mg * kD;
      GemmProblem p = gemm(xk, sb.qkv_w, Mg, 3 * HD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiRopeBF16;
      p.epi.out = s.qkv;
      p.epi.ldo = 3 * HD;
      p.epi.rope = spatial ? w->rope_spatial : w->rope_temporal;
      p.epi.rope_div = spatial ? 1 : kP;
      p.epi.rope_mod = spatial ? kP : T;
      p.epi.rope_stride = spatial ? kP : OASIS_MAX_FRAMES;
      p.epi.rope_dim = HD;
      OASIS_TRY(gemm_launch(p, st));
      if (spatial)
        OASIS_TRY(attention_full_launch(s.qkv, s.attn, Bg * T, kP, H, st));
      else
        OASIS_TRY(attention_temporal_launch(s.qkv, s.attn, Bg, T, kP, H, st));
      OASIS_TRY(project_scatter(k, s.attn, sb.out_w, HD, "reduce_scatter after O"));
    }
    for (int k = 0; k < C; ++k) {
      OASIS_TRY(await(k));  // chunk k's O rows are summed
      OASIS_TRY(residual_chunk(k, sb.out_b, off + 2 * kD));
      OASIS_TRY(ln_chunk(k, off + 3 * kD, off + 4 * kD));
      OASIS_TRY(to_comm());
      OASIS_TRY(collective(a->all_gather, xn_loc + (size_t)k * Mc * kD, xn + (size_t)k * Mg * kD, (size_t)Mc * kD,
                           OASIS_DTYPE_BF16, "all_gather before FC1"));
      OASIS_TRY(mark(k));
    }
    for (int k = 0; k < C; ++k) {
      OASIS_TRY(await(k));
      GemmProblem p = gemm(xn + (size_t)k * Mg * kD, sb.fc1_w, Mg, 4 * HD, kD, s.splitk, s.splitk_bytes);
      p.epi.mode = kEpiGeluTanhBF16;
      p.epi.out = s.h;
      p.epi.ldo = 4 * HD;
      p.epi.bias = sb.fc1_b;
      OASIS_TRY(gemm_launch(p, st));
      OASIS_TRY(project_scatter(k, s.h, sb.fc2_w, 4 * HD, "reduce_scatter after FC2"));
    }
    for (int k = 0; k < C; ++k) {
      OASIS_TRY(await(k));
      OASIS_TRY(residual_chunk(k, sb.fc2_b, off + 5 * kD));
    }
  }
  // final layer over the owned sessions' last frames, then gather v of all sessions
  const long long foff = (long long)w->num_subblocks * OASIS_ADALN_WIDTH;
  LayerNormParams ln;
  ln.P = kP;
  ln.mod = s.adaln;
  ln.ld_mod = ldm;
  ln.shift_off = foff;
  ln.scale_off = foff + kD;
  ln.rows_out = Bl * kP;
  ln.in_group = (long long)T * kP;
  ln.in_off = (long long)(T - 1) * kP;
  ln.frame_mul = T;
  ln.frame_add = T - 1;
  OASIS_TRY(layernorm_launch(z, xn_loc, ln, st));
  GemmProblem p = gemm(xn_loc, w->final_w, Bl * kP, kOut, kD, s.splitk, s.splitk_bytes);
  p.epi.mode = kEpiF32;
  p.epi.out = a->v_local;
  p.epi.ldo = kOut;
  p.epi.bias = w->final_b;
  OASIS_TRY(gemm_launch(p, st));
  OASIS_TRY(to_comm());
  OASIS_TRY(collective(a->all_gather, a->v_local, a->v_out, (size_t)Bl * kP * kOut, OASIS_DTYPE_F32,
                       "all_gather of v"));
  OASIS_TRY(mark(0));
  return await(0);  // the caller's stream sees v and every collective's buffers released
}

// ---- context caching (precompute_past_state / dit_forward_currentonly) ----

size_t kv_cache_bytes(int B, int Tp) { return (size_t)(OASIS_DIT_SUBBLOCKS / 2) * kv_slot_elems(B, Tp) * 2; }

int precompute_past_impl(const OasisDitWeights* w, const OasisDitArgs* a, void* cache, size_t cache_bytes,
                         cudaStream_t st) {
  OASIS_REQUIRE(w && a, "precompute_past: null argument");
  const int B = a->batch, Tp = a->frames;
  OASIS_REQUIRE(B > 0 && Tp >= 1 && Tp <= 31, "precompute_past: batch=%d frames=%d (need frames in [1, 31])", B, Tp);
  OASIS_REQUIRE(a->z && a->cond && cache, "precompute_past: null tensor");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "precompute_past: num_subblocks");
  if (cache_bytes < kv_cache_bytes(B, Tp))
    return set_error(OASIS_ERR_WORKSPACE, "precompute_past: kv cache %zu bytes < %zu", cache_bytes,
                     kv_cache_bytes(B, Tp));
  Carve c(a->workspace, a->workspace_bytes);
  DitScratch s;
  carve_dit(c, B, Tp, &s);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "precompute_past: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  OASIS_TRY(compute_adaln(w, a->cond, B * Tp, s.silu, s.adaln, s.splitk, s.splitk_bytes, st));
  KvCtx kv;
  kv.mode = kKvSave;
  kv.cache = static_cast<__nv_bfloat16*>(cache);
  kv.past_frames = Tp;
  return dit_blocks(w, B, Tp, a->z, s.adaln, nullptr, 0, s, st, kv);
}

int forward_current_impl(const OasisDitWeights* w, const OasisDitArgs* a, const void* cache, size_t cache_bytes,
                         int Tp, cudaStream_t st) {
  OASIS_REQUIRE(w && a, "forward_current: null argument");
  const int B = a->batch;
  OASIS_REQUIRE(B > 0 && a->frames == 1, "forward_current: batch=%d frames=%d (frames must be 1)", B, a->frames);
  OASIS_REQUIRE(Tp >= 0 && Tp <= 31, "forward_current: past_frames=%d outside [0, 31]", Tp);
  OASIS_REQUIRE(a->z && a->cond && a->v_out && (cache || Tp == 0), "forward_current: null tensor");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "forward_current: num_subblocks");
  if (Tp > 0 && cache_bytes < kv_cache_bytes(B, Tp))
    return set_error(OASIS_ERR_WORKSPACE, "forward_current: kv cache %zu bytes < %zu", cache_bytes,
                     kv_cache_bytes(B, Tp));
  Carve c(a->workspace, a->workspace_bytes);
  DitScratch s;
  carve_dit(c, B, 1, &s);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "forward_current: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  OASIS_TRY(compute_adaln(w, a->cond, B, s.silu, s.adaln, s.splitk, s.splitk_bytes, st));
  KvCtx kv;
  kv.mode = kKvUse;
  kv.cache = static_cast<__nv_bfloat16*>(const_cast<void*>(cache));
  kv.past_frames = Tp;
  return dit_blocks(w, B, 1, a->z, s.adaln, a->v_out, 1, s, st, kv);
}

struct FrameKvScratch {
  float* cond_rows;     // [B Tp + S B, 1024]: context rows, then the generated frame's row per step
  __nv_bfloat16* silu;  // same rows
  float* adaln;         // same rows x (6144 S + 2048)
  float* z_past;        // [B Tp 144, 1024]
  float* z;             // [B 144, 1024]
  float* v;             // [B 144, 64]
  float* latent;        // [B, 576, 16]
  __nv_bfloat16* cache;
  void* shared;         // DiT scratch (context pass, then the per-step pass), later the VAE's
  size_t shared_bytes;
};

size_t carve_frame_kv(Carve& c, int B, int T, int S, FrameKvScratch* f) {
  const int Tp = T - 1;
  const size_t R = (size_t)B * Tp + (size_t)S * B;
  FrameKvScratch d;
  d.cond_rows = c.take<float>(R * kD);
  d.silu = c.take<__nv_bfloat16>(R * kD);
  d.adaln = c.take<float>(R * OASIS_ADALN_ROWS);
  d.z_past = c.take<float>((size_t)B * Tp * kP * kD);
  d.z = c.take<float>((size_t)B * kP * kD);
  d.v = c.take<float>((size_t)B * kP * kOut);
  d.latent = c.take<float>((size_t)B * kVaeTok * 16);
  d.cache = Tp ? c.take<__nv_bfloat16>(kv_cache_bytes(B, Tp) / 2) : nullptr;
  Carve dit(nullptr, 0), vae(nullptr, 0);
  carve_dit(dit, B, Tp > 1 ? Tp : 1, nullptr, false);
  carve_vae(vae, B, nullptr);
  d.shared_bytes = (dit.used > vae.used ? dit.used : vae.used) + 256;
  d.shared = c.take<uint8_t>(d.shared_bytes);
  if (f) *f = d;
  return c.used;
}

// One frame with the context rows computed once (the reference's default path,
// oasis_inference.py:1934-1960): cond is laid out as for generate_frame
// ([steps][B][T][1024]); the context frames use step 0's rows.
int generate_frame_kv_impl(const OasisDitWeights* w, const OasisVaeWeights* vw, const OasisFrameArgs* a,
                           cudaStream_t st) {
  OASIS_REQUIRE(w && a, "generate_frame_kv: null argument");
  const int B = a->batch, T = a->frames, S = a->steps, Tp = T - 1;
  OASIS_REQUIRE(B > 0 && T > 0 && T <= 32, "generate_frame_kv: batch=%d frames=%d", B, T);
  OASIS_REQUIRE(S > 0 && S <= kMaxFrameSteps, "generate_frame_kv: steps=%d outside [1, %d]", S, kMaxFrameSteps);
  OASIS_REQUIRE(a->chunk && a->cond && a->coeffs, "generate_frame_kv: null tensor");
  OASIS_REQUIRE(T == 1 || a->context_z, "generate_frame_kv: frames > 1 needs context_z");
  OASIS_REQUIRE(a->skip_decode || (vw && a->image), "generate_frame_kv: decoding needs VAE weights and an image");
  OASIS_REQUIRE(w->num_subblocks >= 0 && w->num_subblocks <= OASIS_DIT_SUBBLOCKS, "generate_frame_kv: num_subblocks");
  Carve c(a->workspace, a->workspace_bytes);
  FrameKvScratch f;
  carve_frame_kv(c, B, T, S, &f);
  if (!a->workspace || !c.ok())
    return set_error(OASIS_ERR_WORKSPACE, "generate_frame_kv: workspace %zu bytes < %zu", a->workspace_bytes, c.used);
  Carve dc(f.shared, f.shared_bytes);
  DitScratch s;
  carve_dit(dc, B, Tp > 1 ? Tp : 1, &s, false);
  const long long ldm = (long long)w->num_subblocks * OASIS_ADALN_WIDTH + 2 * kD;
  const size_t row = kD * sizeof(float);
  // gather the conditioning rows that are used: context frames (step 0), then the
  // generated frame of every step (rows (i B + b) T + T - 1: one constant stride)
  if (Tp > 0) {
    cudaError_t e = cudaMemcpy2DAsync(f.cond_rows, Tp * row, a->cond, T * row, Tp * row, B, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "generate_frame_kv: cond copy: %s", cudaGetErrorString(e));
  }
  {
    cudaError_t e = cudaMemcpy2DAsync(f.cond_rows + (size_t)B * Tp * kD, row, a->cond + (size_t)Tp * kD, T * row, row,
                                      (size_t)S * B, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "generate_frame_kv: cond copy: %s", cudaGetErrorString(e));
  }
  const int R = B * Tp + S * B;
  OASIS_TRY(compute_adaln(w, f.cond_rows, R, f.silu, f.adaln, s.splitk, s.splitk_bytes, st));
  KvCtx kv;
  kv.cache = f.cache;
  kv.past_frames = Tp;
  if (Tp > 0) {
    cudaError_t e = cudaMemcpyAsync(f.z_past, a->context_z, (size_t)B * Tp * kP * row, cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "generate_frame_kv: context copy: %s", cudaGetErrorString(e));
    kv.mode = kKvSave;
    OASIS_TRY(dit_blocks(w, B, Tp, f.z_past, f.adaln, nullptr, 0, s, st, kv));
  }
  kv.mode = kKvUse;
  for (int i = 0; i < S; ++i) {
    PatchEmbedParams pe;
    pe.rows = B * kP;
    pe.P = kP;
    pe.out_group = kP;
    pe.out_off = 0;
    OASIS_TRY(patch_embed_launch(a->chunk, w->embed_w, w->embed_b, f.z, pe, st));
    OASIS_TRY(dit_blocks(w, B, 1, f.z, f.adaln + ((size_t)B * Tp + (size_t)i * B) * ldm, f.v, 1, s, st, kv));
    const OasisDdimCoeffs& k = a->coeffs[i];
    DdimCoeffs dk{k.at_sqrt, k.one_minus_at_sqrt, k.inv_at_sqrt, k.inv_sigma, k.an_sqrt, k.one_minus_an_sqrt};
    OASIS_TRY(ddim_launch(a->chunk, f.v, dk, (long long)B * kP * kOut, st));
  }
  if (a->skip_decode) return OASIS_OK;
  OASIS_TRY(bridge_launch(a->chunk, f.latent, B, 1.0f / kScalingFactor, st));
  OasisVaeArgs va{B, f.latent, a->image, f.shared, f.shared_bytes};
  return vae_decode_impl(vw, &va, st);
}

}  // namespace
}  // namespace oasis

using namespace oasis;

extern "C" {

const char* oasis_last_error(void) { return g_msg; }

const char* oasis_get_last_error(void) { return g_msg; }

int oasis_device_error(int reset) {
  const int a = read_device_error(reset);
  const int b = read_device_error_tc(reset);
  const int c = read_device_error_peer(reset);
  return a ? a : (b ? b : c);
}

unsigned long long oasis_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* oasis_version(void) { return "oasis_b200 0.1 (sm_100a)"; }

size_t oasis_dit_workspace_size(int batch, int frames) {
  Carve c(nullptr, 0);
  return carve_dit(c, batch, frames, nullptr) + 256;
}

int oasis_dit_forward(const OasisDitWeights* w, const OasisDitArgs* a, oasis_stream_t stream) {
  g_msg[0] = 0;
  return dit_forward_impl(w, a, S(stream));
}

int oasis_ddim_update(float* chunk, const float* v, const OasisDdimCoeffs* c, long long n, oasis_stream_t stream) {
  OASIS_REQUIRE(c, "ddim_update: null coefficients");
  DdimCoeffs k{c->at_sqrt, c->one_minus_at_sqrt, c->inv_at_sqrt, c->inv_sigma, c->an_sqrt, c->one_minus_an_sqrt};
  return ddim_launch(chunk, v, k, n, S(stream));
}

size_t oasis_step_workspace_size(int batch, int frames) {
  return step_ws(batch, frames, nullptr, nullptr, nullptr, nullptr, 0) + 256;
}

int oasis_ddim_step(const OasisDitWeights* w, const OasisStepArgs* a, oasis_stream_t stream) {
  g_msg[0] = 0;
  OASIS_REQUIRE(w && a, "ddim_step: null argument");
  const int B = a->batch, T = a->frames;
  OASIS_REQUIRE(B > 0 && T > 0 && T <= 32, "ddim_step: batch=%d frames=%d", B, T);
  OASIS_REQUIRE(a->chunk && a->cond, "ddim_step: null tensor");
  OASIS_REQUIRE(T == 1 || a->context_z, "ddim_step: frames > 1 needs context_z");
  DitScratch s;
  float *z, *v;
  const size_t need = step_ws(B, T, &s, &z, &v, a->workspace, a->workspace_bytes);
  if (!a->workspace || need > a->workspace_bytes)
    return set_error(OASIS_ERR_WORKSPACE, "ddim_step: workspace %zu bytes < %zu", a->workspace_bytes, need);
  cudaStream_t st = S(stream);
  if (T > 1) {
    const size_t ctx_bytes = (size_t)(T - 1) * kP * kD * sizeof(float);
    cudaError_t e = cudaMemcpy2DAsync(z, (size_t)T * kP * kD * sizeof(float), a->context_z, ctx_bytes, ctx_bytes, B,
                                      cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return set_error(OASIS_ERR_CUDA, "ddim_step: context copy: %s", cudaGetErrorString(e));
  }
  PatchEmbedParams pe;
  pe.rows = B * kP;
  pe.P = kP;
  pe.out_group = (long long)T * kP;
  pe.out_off = (long long)(T - 1) * kP;
  OASIS_TRY(patch_embed_launch(a->chunk, w->embed_w, w->embed_b, z, pe, st));
  OasisDitArgs da{B, T, z, a->cond, v, 1, a->workspace, a->workspace_bytes};
  OASIS_TRY(dit_forward_impl(w, &da, st));
  DdimCoeffs k{a->coeffs.at_sqrt, a->coeffs.one_minus_at_sqrt, a->coeffs.inv_at_sqrt, a->coeffs.inv_sigma,
               a->coeffs.an_sqrt, a->coeffs.one_minus_an_sqrt};
  return ddim_launch(a->chunk, v, k, (long long)B * kP * kOut, st);
}

int oasis_patch_embed(const OasisDitWeights* w, const float* patches, int rows, float* z, long long out_group,
                      long long out_off, oasis_stream_t stream) {
  OASIS_REQUIRE(w, "patch_embed: null weights");
  PatchEmbedParams pe;
  pe.rows = rows;
  pe.P = kP;
  pe.out_group = out_group;
  pe.out_off = out_off;
  return patch_embed_launch(patches, w->embed_w, w->embed_b, z, pe, S(stream));
}

int oasis_bridge_unpatchify(const float* chunk, float* latent, int batch, oasis_stream_t stream) {
  return bridge_launch(chunk, latent, batch, 1.0f / kScalingFactor, S(stream));
}

size_t oasis_vae_workspace_size(int batch) {
  Carve c(nullptr, 0);
  return carve_vae(c, batch, nullptr) + 256;
}

int oasis_vae_decode(const OasisVaeWeights* w, const OasisVaeArgs* a, oasis_stream_t stream) {
  g_msg[0] = 0;
  return vae_decode_impl(w, a, S(stream));
}

size_t oasis_vae_encoder_workspace_size(int batch) {
  if (batch <= 0) return 0;
  Carve c(nullptr, 0);
  return carve_vae_enc(c, batch, nullptr, nullptr, nullptr) + 256;
}

int oasis_vae_encode(const OasisVaeEncoderWeights* w, const OasisVaeEncodeArgs* a, oasis_stream_t stream) {
  g_msg[0] = 0;
  return vae_encode_impl(w, a, S(stream));
}

size_t oasis_frame_workspace_size(int batch, int frames, int steps) {
  Carve c(nullptr, 0);
  return carve_frame(c, batch, frames, steps, nullptr) + 256;
}

int oasis_generate_frame(const OasisDitWeights* w, const OasisVaeWeights* vw, const OasisFrameArgs* a,
                         oasis_stream_t stream) {
  g_msg[0] = 0;
  return generate_frame_impl(w, vw, a, S(stream));
}

size_t oasis_tp_workspace_size(int batch, int frames, int heads) {
  if (batch <= 0 || frames <= 0 || heads <= 0) return 0;
  Carve c(nullptr, 0);
  return carve_tp(c, batch, frames, heads, nullptr) + 256;
}

int oasis_dit_forward_tp(const OasisDitWeights* shard, const OasisTpArgs* a, oasis_stream_t stream) {
  g_msg[0] = 0;
  return tp_forward_impl(shard, a, S(stream));
}

size_t oasis_tp_sp_workspace_size(int batch, int frames, int heads, int world) {
  if (world < 1 || heads < 1 || batch < world || batch % world) return 0;
  Carve c(nullptr, 0);
  return carve_tp_sp(c, batch, frames, heads, world, nullptr);
}

int oasis_dit_forward_tp_sp(const OasisDitWeights* shard, const OasisTpSpArgs* a, oasis_stream_t stream) {
  return tp_sp_forward_impl(shard, a, S(stream));
}

size_t oasis_kv_cache_size(int batch, int past_frames) {
  if (batch <= 0 || past_frames <= 0) return 0;
  return kv_cache_bytes(batch, past_frames);
}

int oasis_dit_precompute_past(const OasisDitWeights* w, const OasisDitArgs* a, void* kv_cache, size_t kv_cache_bytes,
                              oasis_stream_t stream) {
  g_msg[0] = 0;
  return precompute_past_impl(w, a, kv_cache, kv_cache_bytes, S(stream));
}

int oasis_dit_forward_current(const OasisDitWeights* w, const OasisDitArgs* a, const void* kv_cache,
                              size_t kv_cache_bytes, int past_frames, oasis_stream_t stream) {
  g_msg[0] = 0;
  return forward_current_impl(w, a, kv_cache, kv_cache_bytes, past_frames, S(stream));
}

size_t oasis_frame_kv_workspace_size(int batch, int frames, int steps) {
  Carve c(nullptr, 0);
  return carve_frame_kv(c, batch, frames, steps, nullptr) + 256;
}

int oasis_generate_frame_kv(const OasisDitWeights* w, const OasisVaeWeights* vw, const OasisFrameArgs* a,
                            oasis_stream_t stream) {
  g_msg[0] = 0;
  return generate_frame_kv_impl(w, vw, a, S(stream));
}

int oasis_gemm(const OasisGemmArgs* a, oasis_stream_t stream) {
  OASIS_REQUIRE(a, "gemm: null args");
  GemmProblem p;
  p.A = a->a;
  p.lda = a->lda ? a->lda : a->k;
  p.W = a->w;
  p.M = a->m;
  p.N = a->n;
  p.K = a->k;
  p.epi.mode = a->mode;
  p.epi.out = a->out;
  p.epi.ldo = a->ldo ? a->ldo : a->n;
  p.epi.bias = a->bias;
  p.epi.resid = a->resid;
  p.epi.ldr = a->ldr ? a->ldr : a->n;
  p.epi.gate = a->gate;
  p.epi.ldg = a->ldg;
  p.epi.rows_per_frame = a->rows_per_frame > 0 ? a->rows_per_frame : 1;
  p.epi.rope = a->rope;
  p.epi.rope_div = a->rope_div > 0 ? a->rope_div : 1;
  p.epi.rope_mod = a->rope_mod > 0 ? a->rope_mod : 1;
  p.epi.rope_dim = a->rope_dim > 0 ? a->rope_dim : 1024;
  p.epi.rope_stride = a->rope_stride > 0 ? a->rope_stride : p.epi.rope_mod;
  p.block_n = a->block_n;
  p.splits = a->splits;
  p.workspace = a->workspace;
  p.workspace_bytes = a->workspace_bytes;
  p.ln.out = a->ln_out;
  p.ln.mod = a->ln_mod;
  p.ln.ld_mod = a->ln_ld_mod;
  p.ln.shift_off = a->ln_shift_off;
  p.ln.scale_off = a->ln_scale_off;
  p.ln.eps = a->ln_eps > 0 ? a->ln_eps : 1e-6f;
  OASIS_REQUIRE(a->mode >= 0 && a->mode <= kEpiGatedResidLN, "gemm: mode %d unknown", a->mode);
  return gemm_launch(p, S(stream));
}

size_t oasis_gemm_workspace_size(int m, int n, int k) { return gemm_workspace_bytes(m, n, k); }

int oasis_gemm_plan(int m, int n, int k, int mode, int block_n, int splits, int* bn_out, int* splits_out,
                    int* pair_out, size_t* splitk_bytes_out) {
  OASIS_REQUIRE(mode >= kEpiF32 && mode <= kEpiGatedResidLN, "gemm_plan: mode=%d", mode);
  return gemm_plan(m, n, k, mode, block_n, splits, bn_out, splits_out, pair_out, splitk_bytes_out);
}

int oasis_layernorm(const OasisLayerNormArgs* a, oasis_stream_t stream) {
  OASIS_REQUIRE(a, "layernorm: null args");
  LayerNormParams p;
  p.rows_out = a->rows_out;
  p.P = a->P > 0 ? a->P : 1;
  p.in_group = a->in_group ? a->in_group : p.P;
  p.in_off = a->in_off;
  p.frame_mul = a->frame_mul ? a->frame_mul : 1;
  p.frame_add = a->frame_add;
  p.eps = a->eps > 0 ? a->eps : 1e-6f;
  p.mod = a->mod;
  p.ld_mod = a->ld_mod;
  p.shift_off = a->shift_off;
  p.scale_off = a->scale_off;
  p.affine_w = a->affine_w;
  p.affine_b = a->affine_b;
  return layernorm_launch(a->x, static_cast<__nv_bfloat16*>(a->y), p, S(stream));
}

int oasis_silu_bf16(const float* x, void* y, long long n, oasis_stream_t stream) {
  return silu_bf16_launch(x, static_cast<__nv_bfloat16*>(y), n, S(stream));
}

int oasis_attention_spatial(const void* qkv, void* out, int groups, int seq, int heads, oasis_stream_t stream) {
  return attention_full_launch(static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), groups,
                               seq, heads, S(stream));
}

int oasis_attention_temporal(const void* qkv, void* out, int batch, int frames, int heads, oasis_stream_t stream) {
  return attention_temporal_launch(static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), batch,
                                   frames, kP, heads, S(stream));
}

int oasis_attention_temporal_cached(const void* past_qkv, const void* cur_qkv, void* out, int batch, int past_frames,
                                    int heads, oasis_stream_t stream) {
  return attention_temporal_cached_launch(static_cast<const __nv_bfloat16*>(past_qkv),
                                          static_cast<const __nv_bfloat16*>(cur_qkv), static_cast<__nv_bfloat16*>(out),
                                          batch, past_frames, kP, heads, S(stream));
}

int oasis_attention_tc(const void* qkv, void* out, int groups, int seq, int heads, oasis_stream_t stream) {
  return attention_tc_launch(static_cast<const __nv_bfloat16*>(qkv), static_cast<__nv_bfloat16*>(out), groups, seq,
                             heads, S(stream));
}

int oasis_gated_residual(float* z, const float* x, const float* bias, const float* gate, long long ldg,
                         int rows_per_frame, int rows, oasis_stream_t stream) {
  return gated_residual_launch(z, x, bias, gate, ldg, rows_per_frame, rows, S(stream));
}

int oasis_post_quant(const float* latent, const float* w, const float* b, float* z, int rows, oasis_stream_t stream) {
  return post_quant_launch(latent, w, b, z, rows, S(stream));
}

}  // extern "C"
