/*
 * gfxinfer-b200 C ABI.
 *
 * A thin, allocation-free launch layer over hand-written sm_100a kernels. It
 * replaces the reference engine's HIP launchers (include/gfxinfer/lowbit_gemv.h,
 * include/gfxinfer/qwen_ops.h) and device layer (src/device.cpp). Conventions:
 *
 *  - Every entry point returns a gfxb_status whose values mirror the
 *    reference's ErrorCode (include/gfxinfer/status.h:11-20); the message of
 *    the last failure on the calling thread is gfxb_last_error_message().
 *  - Pointers are device pointers owned by the caller unless stated otherwise;
 *    fp16 buffers are IEEE binary16 bit patterns (uint16_t), bf16 likewise.
 *  - `stream` is a cudaStream_t passed as void*. Launchers never synchronise.
 *  - Validation happens on the host before any launch and reports
 *    GFXB_INVALID_ARGUMENT / GFXB_UNSUPPORTED, as the reference launchers do.
 */
#ifndef GFXB_GFXB_H
#define GFXB_GFXB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Mirrors gfxinfer::ErrorCode (status.h:11-20); hip_error becomes cuda_error. */
typedef enum {
  GFXB_OK = 0,
  GFXB_INVALID_ARGUMENT = 1,
  GFXB_IO_ERROR = 2,
  GFXB_CORRUPT_ARTIFACT = 3,
  GFXB_UNSUPPORTED = 4,
  GFXB_CUDA_ERROR = 5,
  GFXB_OUT_OF_MEMORY = 6,
  GFXB_INTERNAL = 7
} gfxb_status;

/* Weight formats: the reference Quantization values (artifact.h:22-29). */
enum { GFXB_W2 = 1, GFXB_W3 = 2, GFXB_W4 = 3 };

const char* gfxb_last_error_message(void);
int gfxb_abi_version(void);

/* ---- device layer (replaces src/device.cpp:37-90) ------------------------- */
typedef struct {
  int index;
  int compute_major;
  int compute_minor;
  int multiprocessors;
  uint64_t global_memory_bytes;
  char name[128];
} gfxb_device_info;

/* Fails with GFXB_UNSUPPORTED unless the device is sm_100 (B200). Replaces
 * require_gfx1200_device (device.cpp:65-90). */
int gfxb_require_sm100_device(int device_index, gfxb_device_info* info);

/* ---- weight layout ---------------------------------------------------------
 * B200 tiled layout ("b200"): codes [N/16][K/128][block], one block per
 * 16-row x 128-column tile-group, BITS*256 bytes, lane-major so each of a
 * warp's 32 lanes reads its tensor-core fragment with one or two 16-byte
 * loads. Scales [N/16][K/128][16] fp16, the gfx12 tiled scale order
 * (quantization.cpp:311-314). Same byte count as the reference layouts. */

/* Reference row-major packed codes (quantization.cpp:94-124) -> b200 codes. */
int gfxb_repack_rowmajor_to_b200(int format, const uint8_t* rowmajor_codes, uint8_t* b200_codes,
                                 size_t rows, size_t columns, void* stream);
/* Reference gfx12 tiled codes (quantization.cpp:253-318) -> b200 codes. */
int gfxb_repack_gfx12_to_b200(int format, const uint8_t* gfx12_codes, uint8_t* b200_codes,
                              size_t rows, size_t columns, void* stream);
/* Row-major fp16 scales [N][K/128] -> tiled [N/16][K/128][16]. */
int gfxb_tile_scales(const uint16_t* rowmajor_scales, uint16_t* tiled_scales, size_t rows,
                     size_t columns, void* stream);

/* ---- activation packs --------------------------------------------------------
 * The B200 GEMVs read activations as a pack: int8 codes in mma-fragment order
 * [B][K] (within each 128-group the 32 bytes a lane feeds to the tensor core
 * are contiguous), fp16 group scales [B][K/128] and int32 group code sums
 * [B][K/128]. Quantization is the reference's A4/A8 rule
 * (lowbit_gemv.hip:373-436): scale = fp16(amax/7 or amax/127), code =
 * clamp(rint(x/scale)). `packed_a4` (optional, A4 only) additionally receives
 * the reference's packed-nibble layout [B][K/2]. */
int gfxb_pack_activation(int activation_bits, const uint16_t* input, int8_t* codes,
                         uint16_t* scales, int32_t* sums, uint8_t* packed_a4, size_t columns,
                         unsigned batch, void* stream);

/* ---- GEMV -------------------------------------------------------------------
 * y[b][n] = sum over groups g (ascending) of fp32 fma( int32 dot_g,
 * ws[n][g] * as[b][g] ) (lowbit_gemv.hip:490-537): bit-identical to the
 * reference arithmetic. Output batch-major [B][N], fp32 or fp16. */
typedef struct {
  const uint8_t* codes;    /* b200 layout */
  const uint16_t* scales;  /* tiled fp16 */
  void* output;            /* [B][rows], fp32 or fp16 */
  size_t rows;             /* multiple of 16 */
  int output_f16;          /* 0: fp32, 1: fp16 (launch_gfx12_i4_gemm_half) */
} gfxb_gemv_matrix;

/* One launch for 1..4 matrices that share K, format and input (replaces
 * launch_gfx12_i4_gemm / _half / _fused and launch_gfx12_i8_gemm when the
 * weights are in the b200 layout). batch in [1, 32]. */
int gfxb_lowbit_gemv(int format, const gfxb_gemv_matrix* matrices, unsigned matrix_count,
                     const int8_t* act_codes, const uint16_t* act_scales,
                     const int32_t* act_sums, size_t columns, unsigned batch, void* stream);

/* ---- reference-layout drop-ins (lowbit_gemv.h:79-170) ------------------------ */
int gfxb_quantize_activation_i4(const uint16_t* input, uint8_t* packed_output, uint16_t* scales,
                                size_t columns, unsigned batch, void* stream);
int gfxb_quantize_activation_i8(const uint16_t* input, int8_t* quantized_output,
                                uint16_t* scales, size_t columns, unsigned batch, void* stream);
/* Replaces launch_gfx12_i4_gemm (lowbit_gemv.h:100-111): gfx12 tiled weights
 * (W3 in the sequential 3-bit fragment order), packed A4 activations. */
int gfxb_gfx12_i4_gemm(int format, const uint8_t* tiled_weights,
                       const uint16_t* tiled_weight_scales, const uint8_t* packed_activations,
                       const uint16_t* activation_scales, float* output, size_t rows,
                       size_t columns, unsigned batch, int sequential_w3, void* stream);
/* Replaces launch_gfx12_i8_gemm (lowbit_gemv.h:147-157); also accepts W3. */
int gfxb_gfx12_i8_gemm(int format, const uint8_t* tiled_weights,
                       const uint16_t* tiled_weight_scales, const int8_t* quantized_activations,
                       const uint16_t* activation_scales, float* output, size_t rows,
                       size_t columns, unsigned batch, void* stream);

#ifdef __cplusplus
}
#endif
#endif
