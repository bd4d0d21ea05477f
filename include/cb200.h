/*
 * cb200.h — C ABI of the B200 (sm_100a) quantized-GEMM library.
 *
 * The library implements the quantized-GEMM hot path of the cache-barrier
 * study (W8A8 per-token x per-channel INT8 GEMM, W4A16 int4 group-dequant GEMM,
 * batched INT4 BMM, packed W4A4 GEMM) as hand-written CUDA for sm_100a
 * (TMA + tcgen05 + TMEM). Every entry point:
 *   - takes plain device pointers, sizes and element strides (no framework types);
 *   - enqueues its work on the caller's stream and returns without a host sync;
 *   - allocates no device memory: split-K scratch lives in a caller-owned
 *     workspace whose size cb_workspace_bytes() reports. A workspace must be
 *     zero-filled once when it is allocated; the kernels leave it zeroed again;
 *   - returns a cb_status code and never aborts the process.
 * A workspace may be used by one stream at a time. Calls that share a workspace
 * on different streams without ordering race.
 *
 * Reference interfaces (paths inside the cache-barrier repository) are cited
 * beside each entry point.
 */
#ifndef CB200_H
#define CB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define CB_API __attribute__((visibility("default")))
#else
#define CB_API
#endif

/* Same handle as cudaStream_t / CUstream. NULL is the legacy default stream. */
typedef struct CUstream_st* cb_stream_t;

/* ---- status codes ------------------------------------------------------- */
enum cb_status {
  CB_OK = 0,
  CB_ERR_INVALID_ARG = 1,    /* null pointer where one is required, negative size */
  CB_ERR_SHAPE = 2,          /* a dimension violates a kernel constraint */
  CB_ERR_DTYPE = 3,          /* unsupported dtype code or dtype combination */
  CB_ERR_ALIGNMENT = 4,      /* pointer or row stride not 16-byte aligned (TMA rule) */
  CB_ERR_STRIDE = 5,         /* innermost dimension not contiguous */
  CB_ERR_WORKSPACE = 6,      /* workspace missing or smaller than cb_workspace_bytes() */
  CB_ERR_CUDA = 7,           /* a CUDA runtime/driver call failed */
  CB_ERR_DEVICE_TIMEOUT = 8, /* a bounded device-side wait expired (see cb_workspace_status) */
  CB_ERR_UNSUPPORTED = 9,    /* no kernel for this device or layout */
  CB_ERR_TOO_LARGE = 10      /* size beyond a documented maximum */
};

/* ---- dtype codes -------------------------------------------------------- */
enum cb_dtype {
  CB_DTYPE_F16 = 0,
  CB_DTYPE_BF16 = 1,
  CB_DTYPE_F32 = 2,
  CB_DTYPE_I8 = 3,
  CB_DTYPE_U8 = 4,
  CB_DTYPE_I32 = 5
};

/* ---- operation codes (for cb_workspace_bytes) --------------------------- */
enum cb_op { CB_OP_W8A8 = 0, CB_OP_W4A16 = 1, CB_OP_W4A4 = 2, CB_OP_NVFP4 = 3 };

/* ---- int4 weight layouts ------------------------------------------------ */
enum cb_w4_layout {
  /* uint8 [batch, K/2, N]: byte (k/2, n) = q[2i] & 0xF | q[2i+1] << 4, two's
     complement nibbles. profiling/bench_l2_barrier.py:92-99 (quantize_weights_int4). */
  CB_W4_REF_U8_KN = 0,
  /* int32 [batch, K/8, N]: nibble j (bits 4j..4j+3) of word (k/8, n) holds q[8*(k/8)+j]. */
  CB_W4_I32_K8N = 1,
  /* Kernel-native tiled layout, uint8 [batch, ceil(N/128), ceil(K/128), 128, 64]:
     one contiguous 8 KiB tile per (128 rows of N) x (128 of K), zero padded.
     Row r of a tile is 64 bytes = four 16-byte chunks; chunk j (k = 32j..32j+31)
     is stored at chunk position j ^ ((r >> 1) & 3). Each 32-bit word holds 8
     consecutive k as nibbles in the order k0,k2,k4,k6,k1,k3,k5,k7. */
  CB_W4_NATIVE = 2
};

/* Human-readable name of a status code (static string). */
CB_API const char* cb_status_str(int status);

/* Library ABI version: major * 10000 + minor * 100 + patch. */
CB_API int cb_version(void);

/* Number of SMs the kernels size their grids for on the current device
   (0 when no device is visible). */
CB_API int cb_device_sm_count(void);

/* Workspace bytes needed by op for a GEMM of `batch` x [M x K] x [K x N]. */
CB_API size_t cb_workspace_bytes(int op, int64_t batch, int64_t M, int64_t N, int64_t K);

/* Copies the workspace status word to *device_status after synchronizing the
   stream. Returns CB_ERR_DEVICE_TIMEOUT if a kernel recorded an expired wait
   (and then clears the word and the workspace's arrival counters, which a
   kernel that gave up a wait may leave behind), CB_OK otherwise. */
CB_API int cb_workspace_status(void* workspace, int* device_status, cb_stream_t stream);

/* Failure-detection test hook (no counterpart in the reference). With a
   nonzero limit_ns, every later W8A8 GEMM launch (all W8A8 entry points and
   the W4A4 path) makes one epilogue thread per CTA wait, bounded by limit_ns,
   on a workspace word that nothing sets: the wait expires, the kernel records
   CB_DEVERR_TIMEOUT in its status word and every role of the CTA takes its
   abort path (skips its remaining work, drains its copies and MMAs, frees its
   tensor memory), so the GPU context stays usable and the caller sees the
   timeout through cb_workspace_status / cb_w8a8_noalloc_status. The output of
   such a call is undefined. 0 (the default) turns the hook off. Process-wide;
   for tests only. */
CB_API void cb_debug_force_wait_timeout(uint64_t limit_ns);

/* Split-K test hook (no counterpart in the reference). A tile whose k-blocks
   are split over several CTAs is normally reduced by its first contributor,
   which polls (for at most 10 us) until the others have published their
   parts; when they have not (CTAs that were not resident together), every
   contributor publishes and the last one to arrive reduces the tile. With
   on != 0 the poll is skipped, so every later W8A8 / FP8 / W4A4 / W4A16 /
   NVFP4 GEMM launch takes the last-arriver path for every cut tile; both
   paths sum the parts in the same order, so outputs are bit-identical.
   Process-wide; for tests only. */
CB_API void cb_debug_force_last_arriver(int on);

/* ---- activation quantization ------------------------------------------- */
/* Per-(batch, row) symmetric int8: scale = max(amax/127, 1e-8),
   q = trunc(a/scale + 0.5*sign(a)) (round half away from zero), IEEE-rounded
   fp32 division. Replaces _quant_act_kernel / quantize_acts_w8
   (profiling/w8a8/w8a8_bmm.py:21-41, 92-106).
   a: [batch, M, K] f16 or bf16, K contiguous, strides in elements.
   q: [batch, M, K] int8, K contiguous. scale: fp32, scale[b * scale_stride_b + m]. */
CB_API int cb_quant_act_i8(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_stride_b,
                    int64_t a_stride_m, int8_t* q, int64_t q_stride_b, int64_t q_stride_m, float* scale,
                    int64_t scale_stride_b, cb_stream_t stream);

/* ---- W8A8 INT8 GEMM ----------------------------------------------------- */
/* out[b, m, n] = cvt( (float)acc[b, m, n] * a_scale[b, m] * w_scale[b, n] ),
   acc = sum_k aq[b, m, k] * w[b, n, k] in int32 (bit exact).
   Replaces _w8a8_bmm_kernel / w8a8_bmm (profiling/w8a8/w8a8_bmm.py:44-81, 118-140).
   aq: int8 [batch, M, K], K contiguous.
   w : int8 [batch, N, K], K contiguous (K-major; the reference's [batch, K, N]
       weight viewed transposed — see cb_repack_w8_kmajor).
   out: [batch, M, N] f16 / bf16 / f32, N contiguous.
   acc_out: optional int32 [batch, M, N] (same strides as out) receiving the raw
       accumulators; NULL to skip.
   strides (elements): {aq_b, aq_m, w_b, w_n, out_b, out_m, a_scale_b, w_scale_b}.
   Constraints: K % 16 == 0, 16-byte aligned aq/w and row strides. */
CB_API int cb_w8a8_gemm(const int8_t* aq, const float* a_scale, const int8_t* w, const float* w_scale, void* out,
                 int out_dtype, int32_t* acc_out, int64_t batch, int64_t M, int64_t N, int64_t K,
                 const int64_t* strides, void* workspace, size_t workspace_bytes, cb_stream_t stream);

/* cb_w8a8_gemm with an optional per-output-channel bias added in fp32 before
   the output rounding:
     out[b, m, n] = cvt( ((float)acc * a_scale[b, m]) * w_scale[b, n] + (float)bias[b * bias_stride_b + n] ).
   This is where vLLM's cutlass_scaled_mm(a, b, scale_a, scale_b, out_dtype, bias)
   adds its bias (in the fp32 epilogue), the call the reference's dense
   harnesses make (profiling/dense_qwen/bench_l2_boundary.py:66-71,
   profiling/dense_qwen/bench_dense_proj.py:113-115). bias: f16 / bf16 / f32,
   NULL for none (then identical to cb_w8a8_gemm). */
CB_API int cb_w8a8_gemm_bias(const int8_t* aq, const float* a_scale, const int8_t* w, const float* w_scale,
                             const void* bias, int bias_dtype, int64_t bias_stride_b, void* out, int out_dtype,
                             int32_t* acc_out, int64_t batch, int64_t M, int64_t N, int64_t K,
                             const int64_t* strides, void* workspace, size_t workspace_bytes, cb_stream_t stream);

/* Dynamic per-token activation quantization followed by the W8A8 GEMM, two
   launches chained with programmatic dependent launch so the GEMM's weight
   stream starts while the quantization runs (one launch for one token of a
   single GEMM with K <= 1024: the GEMV quantizes the row itself, with the same
   arithmetic). Replaces w8a8_bmm_full
   (profiling/w8a8/w8a8_bmm.py:143-149). q_buf / s_buf are caller buffers that
   receive the quantized activations (int8 [batch, M, K] contiguous) and scales
   (fp32 [batch * M]), as the reference's `bufs`, in both cases.
   strides (elements): {a_b, a_m, w_b, w_n, out_b, out_m, w_scale_b}. */
CB_API int cb_w8a8_gemm_dynamic(const void* a, int a_dtype, int8_t* q_buf, float* s_buf, const int8_t* w,
                         const float* w_scale, void* out, int out_dtype, int64_t batch, int64_t M, int64_t N,
                         int64_t K, const int64_t* strides, void* workspace, size_t workspace_bytes,
                         cb_stream_t stream);

/* Allocation-free variant of cb_w8a8_gemm (no counterpart in the reference).
   For callers that cannot allocate device memory (another component owns all of
   it, or a foreign-language binding has no allocator to call): same arguments and
   results as cb_w8a8_gemm, without the workspace. The split-K scratch is an 8 MiB
   device array inside this library, present on every GPU that loads it until the
   process exits; problems needing more scratch than that (on a 148-SM B200: more
   than 32 tokens) return CB_ERR_TOO_LARGE. The first call on a device looks the
   array up with that device current; make it before any stream capture. All
   calls on a device share the array: each clears its counters on its stream
   first, and calls whose kernels overlap on the GPU race. The address lookup
   is cached per device for the life of the process: after a device reset
   (cudaDeviceReset or a primary-context reset) reload the library before
   calling again. A bounded device-side wait that expires is recorded in the
   array's status word, which calls do not clear: read it with
   cb_w8a8_noalloc_status. */
CB_API int cb_w8a8_gemm_noalloc(const int8_t* aq, const float* a_scale, const int8_t* w, const float* w_scale,
                                void* out, int out_dtype, int32_t* acc_out, int64_t batch, int64_t M, int64_t N,
                                int64_t K, const int64_t* strides, cb_stream_t stream);

/* Status of cb_w8a8_gemm_noalloc calls on the current device (no counterpart
   in the reference): synchronizes the stream, copies the scratch array's status
   word to *device_status (nullable) and returns CB_ERR_DEVICE_TIMEOUT if any
   call since the last read recorded an expired wait (then clears the word and
   the array's counters), CB_OK otherwise. The device-side counterpart of
   cb_workspace_status for callers that hold no workspace. */
CB_API int cb_w8a8_noalloc_status(int* device_status, cb_stream_t stream);

/* ---- host-buffer executor (no counterpart in the reference) -------------
   For callers whose activations and results live in host memory (a serving
   loop, a foreign-language binding): one call copies the activations in,
   runs cb_w8a8_gemm_dynamic and copies the result back, all enqueued on the
   executor's own three streams (copy-in, compute, copy-out) with a ring of two
   device buffer sets, so consecutive calls overlap one call's copies with the
   neighbouring calls' kernels. Calls return once the work is enqueued; host
   buffers must stay valid (and the output unread) until cb_exec_synchronize
   or until work ordered after the call by cb_exec_before has completed. Use
   page-locked (pinned) host memory: with pageable memory the copies still
   give the right result but block the calling thread. An executor owns its
   device buffers (grown on demand, which first waits for its work in flight)
   and is not thread-safe: one thread at a time per executor. */
typedef struct cb_exec cb_exec;
CB_API int cb_exec_create(int device, cb_exec** exec);
CB_API void cb_exec_destroy(cb_exec* exec);
/* Work enqueued on the executor after this call waits for the work enqueued on
   `stream` before it. */
CB_API int cb_exec_after(cb_exec* exec, cb_stream_t stream);
/* Work enqueued on `stream` after this call waits for all work the executor
   has enqueued so far (copies back to the host included). */
CB_API int cb_exec_before(cb_exec* exec, cb_stream_t stream);
/* Waits for all of the executor's work; then reads and clears its workspace
   status word like cb_workspace_status (CB_ERR_DEVICE_TIMEOUT if a kernel
   recorded an expired wait). */
CB_API int cb_exec_synchronize(cb_exec* exec, int* device_status);
/* out_host[b, m, n] = w8a8_bmm_full(a_host, w)[b, m, n]: a_host f16/bf16
   [batch, M, K] and out_host [batch, M, N] (f16/bf16/f32) contiguous host
   arrays; w int8 [batch, N, K] (K contiguous) and w_scale fp32 [batch, N] in
   device memory, with element strides w_stride_b, w_stride_n and
   w_scale_stride_b. Same arithmetic and results as cb_w8a8_gemm_dynamic. */
CB_API int cb_exec_w8a8_dynamic_host(cb_exec* exec, const void* a_host, int a_dtype, const int8_t* w,
                                     const float* w_scale, int64_t w_stride_b, int64_t w_stride_n,
                                     int64_t w_scale_stride_b, void* out_host, int out_dtype, int64_t batch,
                                     int64_t M, int64_t N, int64_t K);

/* ---- FP8 (e4m3) W8A8 GEMM ----------------------------------------------- */
/* The reference measures its W8A8 path against vLLM's fp8 cutlass_scaled_mm
   on e4m3 operands (profiling/dense_qwen/bench_l2_boundary.py:54-57, 66-68;
   profiling/dense_qwen/bench_dense_proj.py:40-43, 113-115). These entry points
   give that path on the tcgen05 kind::f8f6f4 tensor cores. */
enum cb_fp8_mode {
  CB_FP8_PER_TOKEN = 0,          /* dynamic, one scale per (batch, row) */
  CB_FP8_PER_TENSOR_DYNAMIC = 1, /* dynamic, one scale per batch entry from its amax */
  CB_FP8_STATIC = 2              /* scale[b * scale_stride_b] given by the caller */
};
/* e4m3 quantization of activations a [batch, M, K] (f16 / bf16, K contiguous):
   dynamic scale = max(amax / 448, 1 / (448 * 512)) (IEEE-rounded division),
   q = e4m3(clamp(a / scale, -448, 448)), round to nearest even. q: uint8 e4m3
   bytes [batch, M, K]; scale: fp32, scale[b * scale_stride_b + m] per token or
   scale[b * scale_stride_b] per tensor. Replaces vllm._custom_ops.scaled_fp8_quant
   (its per-tensor dynamic, per-token dynamic and static modes). */
CB_API int cb_quant_act_fp8(const void* a, int a_dtype, int64_t batch, int64_t M, int64_t K, int64_t a_stride_b,
                            int64_t a_stride_m, uint8_t* q, int64_t q_stride_b, int64_t q_stride_m, float* scale,
                            int64_t scale_stride_b, int mode, cb_stream_t stream);
/* out[b, m, n] = cvt( (acc * a_scale) * w_scale (+ bias[n]) ), acc = sum_k aq * w
   accumulated in fp32 on the tensor cores (e4m3 products are exact in fp32).
   aq: e4m3 [batch, M, K], w: e4m3 [batch, N, K] (K-major), as cb_w8a8_gemm.
   a_scale: per token (a_scale[b * s_ab + m]) or, with a_scale_per_tensor, one
   value per batch entry (a_scale[b * s_ab]); w_scale likewise per channel or
   per tensor. strides (elements): {aq_b, aq_m, w_b, w_n, out_b, out_m,
   a_scale_b, w_scale_b}. Workspace: cb_workspace_bytes(CB_OP_W8A8, ...).
   Replaces vllm._custom_ops.cutlass_scaled_mm on e4m3 operands. */
CB_API int cb_fp8_gemm(const uint8_t* aq, const float* a_scale, int a_scale_per_tensor, const uint8_t* w,
                       const float* w_scale, int w_scale_per_tensor, const void* bias, int bias_dtype, void* out,
                       int out_dtype, int64_t batch, int64_t M, int64_t N, int64_t K, const int64_t* strides,
                       void* workspace, size_t workspace_bytes, cb_stream_t stream);

/* ---- W4A16 int4 group-dequant GEMM / batched INT4 BMM -------------------- */
/* out[b, m, n] = sum_k a[b, m, k] * (q[b, k, n] * s[b, k / group_size, n]).
   Replaces kernel_batched_w4a16_simple / batched_int4_gemm
   (profiling/bench_l2_barrier.py:36-85, 102-125; profiling/int4_batched_gemm.py:130-265;
   profiling/int4_batched_gemm_v2.py:140-260) and generalises the per-channel
   scale (group_size == K) to group_size 128 (or any multiple of 128).
   a: [batch, M, K] f16 or bf16 (K contiguous); the MMA runs in a's dtype.
   w_native: CB_W4_NATIVE layout (see cb_repack_w4).
   scales: [batch, ceil(K/group_size), N] f16 / bf16 / f32, N contiguous.
   out: [batch, M, N] f16 / bf16 / f32, N contiguous.
   strides (elements): {a_b, a_m, s_b, s_g, out_b, out_m}.
   Constraints: K % 8 == 0; group_size % 128 == 0 or group_size >= K. */
CB_API int cb_w4a16_gemm(const void* a, int a_dtype, const uint8_t* w_native, const void* scales, int scale_dtype,
                  int64_t group_size, void* out, int out_dtype, int64_t batch, int64_t M, int64_t N, int64_t K,
                  const int64_t* strides, void* workspace, size_t workspace_bytes, cb_stream_t stream);

/* ---- W4A4 packed int4 GEMM ---------------------------------------------- */
/* Nibble interpretation for cb_w4a4_gemm. */
enum cb_w4a4_mode {
  /* two's complement int4 in [-8, 7]: the function's documented contract
     (kernels/triton_gemm.py:407-411) and its own check (:492-520). */
  CB_W4A4_SIGNED = 0,
  /* what the reference kernel computes: `v - 16` on a uint8 tensor for v >= 8
     (kernels/triton_gemm.py:164-167) wraps to 240..255. */
  CB_W4A4_REF_UINT8_WRAP = 1
};
/* C[m, n] = sum_k A[m, k] * B[k, n] as fp32 (exact integer sums, one rounding).
   Replaces triton_gemm_packed_int4 (kernels/triton_gemm.py:395-485).
   a_packed: uint8 [M, K/2] (byte (m, i) holds k = 2i low, 2i+1 high), row stride lda.
   b_packed: uint8 [K/2, N], row stride ldb. c: fp32 [M, N], row stride ldc.
   The workspace also holds the unpacked 8-bit operands. K % 32 == 0. */
CB_API int cb_w4a4_gemm(const uint8_t* a_packed, const uint8_t* b_packed, float* c, int64_t M, int64_t N, int64_t K,
                        int64_t lda, int64_t ldb, int64_t ldc, int nibble_mode, void* workspace,
                        size_t workspace_bytes, cb_stream_t stream);

/* ---- NVFP4 (e2m1 values, e4m3 scales per 16 elements) ------------------- */
/* The matched-precision W4A4 path the reference runs through vLLM on B200
   (profiling/cuda_validation/bench_moe_nvfp4_native.py:97-108: scaled_fp4_quant,
   run_cutlass_moe_fp4), in vLLM's tensor formats (vllm 0.22.0):
     values: uint8 [rows, K/2], element 2i in the low nibble, 2i+1 in the high;
             nibble = sign << 3 | index into {0, 0.5, 1, 1.5, 2, 3, 4, 6};
     scales: e4m3 bytes, 512-byte atoms of 128 rows x 4 scale columns,
             ceil(rows/128) * ceil(K/64) atoms, byte (r, c) at
             ((r/128) * ceil(K/64) + c/4) * 512 + (r%32) * 16 + ((r%128)/32) * 4 + c%4.
   Quantization of x [rows, K] (f16 / bf16, row stride x_stride elements) with a
   per-tensor global scale gs (one fp32 on the device), as vLLM's
   ref_nvfp4_quant (nvfp4_emulation_utils.py:439-453):
     s = e4m3(gs * amax_block * (1/6)), o = 1 / (s * (1/gs)), q = e2m1(clamp(x * o, +-6)),
   round to nearest even throughout; padding scale bytes are written as 0.
   q: [rows, K/2] with row stride q_stride bytes; sf: ceil(rows/128)*128 * K/16 bytes
   (K % 64 == 0). Replaces vllm._custom_ops.scaled_fp4_quant(x, gs). */
CB_API int cb_nvfp4_quantize(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t x_stride,
                             const float* global_scale, uint8_t* q, int64_t q_stride, uint8_t* sf,
                             cb_stream_t stream);
/* out[m, n] = alpha * sum_k A[m, k] * B[n, k], fp32 accumulation on the
   tensor cores' block-scaled FP4 path (tcgen05.mma kind::mxf4nvf4).
   a: activations [M, K/2] (row stride a_stride bytes), a_sf their scales;
   b: weights [N, K/2] (row stride b_stride bytes), b_sf their scales;
   alpha: one fp32 on the device (1 / (gs_a * gs_b) for vLLM-quantized operands);
   out: [M, N] f16 / bf16 / f32, row stride out_stride elements. K % 64 == 0;
   16-byte aligned operands and strides. Workspace from
   cb_workspace_bytes(CB_OP_NVFP4, 1, M, N, K). Replaces
   vllm._custom_ops.cutlass_scaled_fp4_mm(a, b, a_sf, b_sf, alpha, out_dtype). */
CB_API int cb_nvfp4_gemm(const uint8_t* a, const uint8_t* a_sf, const uint8_t* b, const uint8_t* b_sf,
                         const float* alpha, void* out, int out_dtype, int64_t M, int64_t N, int64_t K,
                         int64_t a_stride, int64_t b_stride, int64_t out_stride, void* workspace,
                         size_t workspace_bytes, cb_stream_t stream);

/* ---- weight preparation (offline, device-side) -------------------------- */
/* Repack int4 weights from CB_W4_REF_U8_KN or CB_W4_I32_K8N into CB_W4_NATIVE.
   src strides are the dense strides of the source layout; dst must hold
   cb_w4_native_bytes(batch, K, N) bytes. */
CB_API int cb_repack_w4(const void* src, int src_layout, uint8_t* dst_native, int64_t batch, int64_t K, int64_t N,
                 cb_stream_t stream);
CB_API size_t cb_w4_native_bytes(int64_t batch, int64_t K, int64_t N);

/* Transpose int8 weights [batch, K, N] (N contiguous, the reference layout of
   quantize_weights_w8, profiling/w8a8/w8a8_bmm.py:84-89) into [batch, N, K]. */
CB_API int cb_repack_w8_kmajor(const int8_t* src_kn, int8_t* dst_nk, int64_t batch, int64_t K, int64_t N,
                        cb_stream_t stream);

/* Fused RMSNorm -> dynamic per-token int8 quantization (no counterpart kernel in
   the reference, which measures this fusion with library ops:
   profiling/mechanisms/RESULTS.md:17). Per row of x [rows, H] (f16/bf16, row
   stride x_sm): r = 1/sqrt(sum x^2 / H + eps) in fp32; y = cvt(x * r * w) in x's
   dtype; then scale and q exactly as cb_quant_act_i8 on y. weight: [H] f16, bf16
   or f32. y_out (nullable, row stride y_sm) receives y. */
CB_API int cb_rmsnorm_quant_i8(const void* x, int x_dtype, const void* weight, int w_dtype, float eps, int64_t rows,
                               int64_t H, int64_t x_sm, int8_t* q, int64_t q_sm, float* scale, void* y_out,
                               int64_t y_sm, cb_stream_t stream);

/* ---- One-shot all-reduce over NVLink peer memory (tensor-parallel projections) ----
 * No counterpart in the reference, which has no multi-GPU code: it replaces the
 * NCCL all-reduce after the row-parallel O and down projections of a
 * tensor-parallel decoder for small [T, hidden] 16-bit partials.
 *
 * Setup (once per rank, all ranks alike): cb_symm_alloc(cb_symm_bytes(world,
 * slot_elems)) gives this rank's zeroed symmetric area; cb_ipc_get_handle
 * exports it as a 64-byte CUDA IPC handle, the host exchanges handles, and
 * cb_ipc_open_handle maps every peer's area. cb_peer_allreduce(in, out, elems,
 * dtype, areas[world], rank, world, slot_elems, status, stream) then sums the
 * world partials `in` into `out` on every rank (same values on all ranks, fp32
 * sums in rank order). Every rank must issue the same sequence of calls with the
 * same element counts. A peer that never joins makes the call return after about
 * a second with CB_DEVERR_TIMEOUT set in *status (a device int). */
CB_API size_t cb_symm_bytes(int world, int64_t slot_elems);
CB_API int cb_symm_alloc(size_t bytes, void** ptr);
CB_API int cb_symm_free(void* ptr);
CB_API int cb_ipc_get_handle(const void* dev_ptr, void* handle_out /* 64 bytes */);
CB_API int cb_ipc_open_handle(const void* handle_in /* 64 bytes */, void** peer_ptr);
CB_API int cb_ipc_close_handle(void* peer_ptr);
CB_API int cb_peer_allreduce(const void* in, void* out, int64_t elems, int dtype, void* const* symm_areas, int rank,
                             int world, int64_t slot_elems, int* status, cb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* CB200_H */
