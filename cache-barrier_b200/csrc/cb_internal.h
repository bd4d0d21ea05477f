// Host-side internals shared by the kernel launchers and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "cb200.h"

namespace cb {

constexpr int kMaxStages = 16;
// Workspace header: word 0 is the status word; word 1 is never written (the
// failure-detection test hook waits on it); the rest is padding.
constexpr size_t kWsHeader = 256;

// Wait limit of the failure-detection test hook (0 = off), set by
// cb_debug_force_wait_timeout and read by the W8A8 launcher.
unsigned long long debug_wait_ns();
// Split-K test hook (cb_debug_force_last_arriver): cut tiles skip the first
// contributor's poll, so every one is reduced by its last arriver.
bool debug_force_last_arriver();

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// SM count of the current device (cached per device); 0 if no device.
int sm_count();

// Token tile (MMA N) for M tokens: 16, 32, 64, 128 or (max_tile permitting) 256.
inline int token_tile(int64_t M, int max_tile = 256) {
  if (M <= 16) return 16;
  if (M <= 32) return 32;
  if (M <= 64) return 64;
  if (M <= 128 || max_tile <= 128) return 128;
  return 256;
}

// Split-K scratch carved out of the caller's workspace.
struct Workspace {
  int* status;
  int* counters;
  void* partials;
};

// Workspace layout (fixed, so calls of different shapes that share one
// workspace agree on it): [status word + padding][kMaxGrid arrival counters]
// [2 partial slots per CTA].
constexpr int kMaxGrid = 1024;
constexpr size_t kWsCounters = kMaxGrid * sizeof(int);

inline size_t workspace_need(int grid, size_t slot_bytes) {
  return kWsHeader + kWsCounters + 2 * static_cast<size_t>(grid) * slot_bytes;
}

// Stream-K grid: one CTA per SM, but at least TN / 16 (and min_kb_per_cta)
// k-blocks per CTA, so wide token tiles are not cut into many small ranges
// (every cut tile is summed by one CTA from TN * 128 * 4-byte partials of all
// its contributors). Neither minimum exceeds the k-blocks of one tile: a range
// of whole tiles cuts nothing, and with short K (one k-block per tile) every
// SM then gets tiles.
inline int stream_k_grid(long long total_kb, int sms, int TN, int kb_per_tile, int min_kb_per_cta = 1) {
  long long per_cta = TN >= 32 ? TN / 16 : 1;
  if (per_cta < min_kb_per_cta) per_cta = min_kb_per_cta;
  if (per_cta > kb_per_tile) per_cta = kb_per_tile;
  long long grid = (total_kb + per_cta - 1) / per_cta;
  const int max_grid = sms < kMaxGrid ? sms : kMaxGrid;
  if (grid > max_grid) grid = max_grid;
  return grid < 1 ? 1 : static_cast<int>(grid);
}

inline Workspace carve_workspace(void* ws, int grid) {
  (void)grid;
  Workspace w;
  char* base = static_cast<char*>(ws);
  w.status = reinterpret_cast<int*>(base);
  w.counters = reinterpret_cast<int*>(base + kWsHeader);
  w.partials = base + kWsHeader + kWsCounters;
  return w;
}

// 3-D tiled tensor map (dims innermost first; strides of dims 1, 2 in elements).
int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_elems, uint64_t stride2_elems, uint32_t box0, uint32_t box1,
                   CUtensorMapSwizzle swizzle);

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? CB_OK : CB_ERR_CUDA; }

// Synchronizing read of the status word at the start of a workspace (or of the
// no-alloc scratch array); on a recorded timeout it clears the word and the
// arrival counters and returns CB_ERR_DEVICE_TIMEOUT.
int read_and_clear_status(void* scratch, int* device_status, cudaStream_t s);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Argument checks shared by the W8A8 entry points (strides as in cb_w8a8_gemm).
int validate_w8a8(const int8_t* aq, const int8_t* w, void* out, int out_dtype, int64_t batch, int64_t M, int64_t N,
                  int64_t K, const int64_t* st);

// ---- launchers (validated arguments) ----
int launch_act_quant(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_sb, int64_t a_sm,
                     int8_t* q, int64_t q_sb, int64_t q_sm, float* scale, int64_t s_sb, cudaStream_t stream);
// e4m3 quantization of activations: mode CB_FP8_PER_TOKEN (scale per row),
// CB_FP8_PER_TENSOR_DYNAMIC (one scale per batch entry, from its amax) or
// CB_FP8_STATIC (scale[b * s_sb] given).
int launch_act_quant_fp8(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_sb, int64_t a_sm,
                         uint8_t* q, int64_t q_sb, int64_t q_sm, float* scale, int64_t s_sb, int mode,
                         cudaStream_t stream);

struct W8A8Launch {
  const int8_t* aq;
  const float* a_scale;
  const int8_t* w;
  const float* w_scale;
  void* out;
  int out_dtype;
  int32_t* acc_out;
  int64_t batch, M, N, K;
  int64_t aq_sb, aq_sm, w_sb, w_sn, out_sb, out_sm, as_sb, ws_sb;
  int raw_f32;            // 1: out = (float)acc, no scales (W4A4 path)
  int unsigned_operands;  // 1: both operands are uint8 (W4A4 reference-wrap mode)
  int fp8;                // 1: both operands are e4m3 fp8 (fp32 accumulators; acc_out unused)
  int scale_per_tensor_a; // 1: a_scale holds one value per batch entry (else one per token)
  int scale_per_tensor_w; // 1: w_scale holds one value per batch entry (else one per output channel)
  const void* bias;       // optional [batch, N] bias (f16/bf16/f32) added in fp32 before rounding
  int bias_dtype;
  int64_t bias_sb;
  void* workspace;
  size_t workspace_bytes;
};
int launch_w8a8(const W8A8Launch& L, cudaStream_t stream);
// One or two tokens per batch entry: the dp4a GEMV kernel (w8a8_gemv.cu); of
// the workspace it uses only the status word.
bool w8a8_gemv_eligible(const W8A8Launch& L);
int launch_w8a8_gemv(const W8A8Launch& L, cudaStream_t stream);
// Dynamic quantization fused into the GEMV (one token of a single GEMM, short
// rows): the kernel quantizes the 16-bit row a itself and stores q / scale to
// L.aq / L.a_scale.
bool w8a8_gemv_dynamic_eligible(const W8A8Launch& L, const void* a, int a_dtype, int64_t a_sm);
int launch_w8a8_gemv_dynamic(const W8A8Launch& L, const void* a, int a_dtype, int64_t a_sm, cudaStream_t stream);
size_t w8a8_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K);

struct W4A16Launch {
  const void* a;
  int a_dtype;
  const uint8_t* w;
  const void* scales;
  int scale_dtype;
  int64_t group_size;
  void* out;
  int out_dtype;
  int64_t batch, M, N, K;
  int64_t a_sb, a_sm, s_sb, s_sg, out_sb, out_sm;
  void* workspace;
  size_t workspace_bytes;
};
int launch_w4a16(const W4A16Launch& L, cudaStream_t stream);
// Weight-stationary variant for long token dimensions and K <= 512 (w4a16_resident.cu).
bool w4a16_resident_eligible(const W4A16Launch& L);
int launch_w4a16_resident(const W4A16Launch& L, cudaStream_t stream);
size_t w4a16_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K);
// One or two tokens: the dp4a GEMV kernel (w4a16_gemv.cu) instead of the
// tensor-core kernel (from four tokens on, the dp4a chains cost more than the
// tensor cores' fixed MMA time: K = N = 8192, T = 4 took 41.9 us against
// 28 us); at most kGemvCtasPerSm CTAs per SM when it splits K.
constexpr int kGemvMaxTokens = 2;
constexpr int kGemvCtasPerSm = 4;
bool w4a16_gemv_eligible(const W4A16Launch& L);
int launch_w4a16_gemv(const W4A16Launch& L, cudaStream_t stream);

// NVFP4 GEMM: out[M, N] = alpha * A[M, K] . B[N, K]^T (nvfp4.cu). a/b: packed
// e2m1 [rows, K/2] with row strides a_sm / b_sn in bytes; a_sf / b_sf: swizzled
// e4m3 scale atoms; alpha: one fp32 on the device.
struct Nvfp4Launch {
  const uint8_t* a;
  const uint8_t* a_sf;
  const uint8_t* b;
  const uint8_t* b_sf;
  const float* alpha;
  void* out;
  int out_dtype;
  int64_t M, N, K;
  int64_t a_sm, b_sn, out_sm;
  void* workspace;
  size_t workspace_bytes;
};
int launch_nvfp4_gemm(const Nvfp4Launch& L, cudaStream_t stream);
int launch_nvfp4_quant(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t x_sm, const float* global_scale,
                       uint8_t* q, int64_t q_sm, uint8_t* sf, cudaStream_t stream);
size_t nvfp4_workspace_bytes(int64_t M);

}  // namespace cb
