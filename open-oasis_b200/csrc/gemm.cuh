// Host-visible declarations for the tcgen05 GEMM family.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace oasis {

// Epilogue variants fused into the GEMM (acc = A . W^T in fp32, +bias[n] first).
enum EpiMode : int {
  kEpiF32 = 0,          // out_f32 = acc + bias
  kEpiBF16 = 1,         // out_bf16 = acc + bias
  kEpiGeluTanhBF16 = 2, // out_bf16 = gelu_tanh(acc + bias)
  kEpiGeluErfBF16 = 3,  // out_bf16 = gelu_erf(acc + bias)
  kEpiGatedResid = 4,   // out_f32 = resid + gate[frame(r), n] * (acc + bias)
  kEpiResid = 5,        // out_f32 = resid + acc + bias
  kEpiRopeBF16 = 6,     // out_bf16 = rope(acc + bias) on the q and k thirds of a qkv row
  kEpiImage = 7,        // VAE predictor: unpatchify 20x20x3 patches into a clamped image
  kEpiGatedResidLN = 8, // kEpiGatedResid, then LayerNorm + adaLN modulate of the new rows (N = 1024):
                        //   ln_out_bf16[r, n] = (z - mean_r) rstd_r ln_mod[f, scale + n] + ln_mod[f, shift + n]
};

struct EpiParams {
  int mode = kEpiF32;
  void* out = nullptr;
  long long ldo = 0;              // elements between output rows
  const float* bias = nullptr;    // [N] or null
  const float* resid = nullptr;   // residual input (may alias out)
  long long ldr = 0;
  const float* gate = nullptr;    // gated residual: gate[(r / rows_per_frame) * ldg + n]
  long long ldg = 0;
  int rows_per_frame = 1;
  const float* rope = nullptr;    // rope[(q * rope_stride + pos) * 4 + {0..3}]: (cos, sin) of pairs 2q, 2q+1
  int rope_div = 1;               // pos = (r / rope_div) % rope_mod
  int rope_mod = 1;
  int rope_stride = 1;            // positions per q row of the table
  int rope_dim = 1024;            // q occupies [0, rope_dim), k [rope_dim, 2 rope_dim)
  int img_grid_w = 32;            // image mode: tokens per patch row
  int img_tokens = 576;           // image mode: tokens per frame
  int img_patch = 20;             // image mode: patch edge in pixels
};

// kEpiGatedResidLN: the next sub-block's LayerNorm fused into the epilogue (kept
// out of EpiParams, whose fields the epilogue holds in registers).
struct LnParams {
  void* out = nullptr;         // bf16 [M, 1024]
  const float* mod = nullptr;  // adaLN table; frame f = r / rows_per_frame
  long long ld_mod = 0;
  long long shift_off = 0;
  long long scale_off = 0;     // (1 + scale) already folded into the table
  float eps = 1e-6f;
};

struct GemmProblem {
  const void* A = nullptr;  // bf16 [M, K], row stride lda elements
  long long lda = 0;
  const void* W = nullptr;  // bf16 [N, K] (nn.Linear layout), row stride K
  int M = 0, N = 0, K = 0;
  EpiParams epi;
  LnParams ln;              // kEpiGatedResidLN only
  int block_n = 0;          // 0 = heuristic, else 32/64/128/256, or 512: 256 x 256 tiles on a CTA pair
  int splits = 0;           // 0 = heuristic, 1 = no split-K
  void* workspace = nullptr;  // split-K partial tiles (may be null -> no split)
  size_t workspace_bytes = 0;
};

// Returns 0 or a negative oasis status code.
int gemm_launch(const GemmProblem& p, cudaStream_t stream);

// Bytes of split-K workspace the heuristic may want for an M x N x K problem.
size_t gemm_workspace_bytes(int M, int N, int K);

// Split-K workspace bytes a launch with this epilogue mode and these overrides
// (0 = heuristic) needs, given that a workspace is passed.
size_t gemm_splitk_bytes(int M, int N, int K, int mode, int block_n, int splits);

// The tile plan gemm_launch uses for such a launch (with a workspace): tile width
// (512 = 256 x 256 tiles on a CTA pair), K splits, pair flag and split-K bytes.
// Returns 0 or a negative status for overrides the launch would reject.
int gemm_plan(int M, int N, int K, int mode, int block_n, int splits, int* bn, int* splits_out, int* pair,
              size_t* splitk_bytes);

int num_sms();

// SMs the persistent kernels (GEMMs, tcgen05 attention) size their grids for:
// num_sms() minus a reserve set on this host thread, which leaves SMs free for
// kernels of another stream (the collectives of overlapped tensor parallelism).
int grid_sms();
void set_sm_reserve(int n);

// 2-D bf16 TMA map with the 128-byte swizzle over a row-major matrix of `outer`
// rows x `inner` columns (row stride `ld` elements), box {box_inner, box_outer}.
int make_tma_bf16_2d(CUtensorMap* map, const void* ptr, long long inner, long long outer, long long ld,
                     int box_inner, int box_outer);

}  // namespace oasis
