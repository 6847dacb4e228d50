// Exact int16 x int16 GEMM on the int8 tensor cores (tcgen05 kind::i8): the
// shared engine of MatmulKernel and ConvKernel jobs.
//
// Each int16 operand arrives split into planes hi = v >> 8 (signed byte) and
// lo = v & 255 (unsigned byte), K-major [batch][rows][Kp] (Kp a multiple of
// 16, zero padded).  Per 128 x 128 output tile three int32 TMEM accumulators
// collect HH = sum a_hi b_hi, MID = sum a_hi b_lo + a_lo b_hi and LL = sum a_lo
// b_lo — exact for K <= 32768 — and the epilogue forms the exact sum
// 2^16 HH + 2^8 MID + LL (+ bias << 8) in int64, applies the job's rule
// (optional int32 wrap, floor >> 8, saturation, optional ReLU / Clip(0,6))
// and stores int16.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "postop.cuh"

namespace corm {

struct GemmJob {
  const int8_t* a_hi;
  const uint8_t* a_lo;
  const int8_t* b_hi;
  const uint8_t* b_lo;
  uint32_t rows, cols, Kp, batch;
  uint32_t a_planes, b_planes;  // 1 (broadcast) or batch
  // B planes: K-major [planes][cols][Kp] (b_mn = 0), or MN-major [planes][K][cols_p]
  // with cols_p = cols rounded up to 16 (b_mn = 1)
  uint32_t b_mn, K, cols_p;
  // K-split partial sums (int64 [split][batch][rows][cols]), gemm_partial_bytes() bytes, or nullptr
  void* partial;
  // epilogue addressing
  int mode;                 // 0: out[b*obs + r*ldc + c]; 1: conv NCHW y[n][pattern(c)][p], r = n*P + p
  int16_t* out;
  uint64_t out_batch_stride;
  uint32_t ldc;
  uint32_t P, y_cn, y_cs, y_gs;
  uint64_t img_stride;      // mode 1: elements per image (out_ch * P)
  const int16_t* bias;      // mode 1 bias per column (raw), or nullptr
  uint32_t bias_rows;       // mode 0: `bias` holds one entry per row (a 1x1 conv run as W x per image)
  uint32_t flags;           // CORM_F_WRAP32 | CORM_F_ACT_RELU | CORM_F_ACT_RELU6
  PostOp post;              // fused VectorOP job on the result (op kPostNone: none)
  // int16 operands split inside the kernel instead of the planes above (a16 != nullptr):
  // A [batch][rows][lda] K-major, B [batch][K][ldb] MN-major (b_mn implied), batch
  // strides in elements (0: shared), 16-byte aligned rows, K and cols multiples of 8.
  // a16 with b16 == nullptr: A split inside the kernel, B from the MN-major planes
  // b_hi / b_lo above (b_mn = 1, cols_p)
  const int16_t* a16;
  const int16_t* b16;
  uint64_t a_bs16, b_bs16;
  uint32_t lda, ldb;
  int* err;                 // status word for the bounded waits; nullptr: the library's per-device word
  // mode 0 with ngroups > 1: output columns split into consecutive groups, group g
  // (gw[g] columns, all but the last a multiple of 32) row-major [batch][rows][gw[g]]
  // at gout[g]; out is then gout[0]
  uint32_t ngroups;
  int16_t* gout[4];
  uint32_t gw[4];
  // gate / up pairs: the columns are 16-column blocks alternating gate, up;
  // out receives MULACT(gate, up) with the shifts ma_sa / ma_sc (the row-ops
  // unit's SiLU(g << sa) u rounded at sc), [batch][rows][cols / 2] at ldc
  uint32_t mulact;
  int32_t ma_sa, ma_sc;
};

constexpr uint32_t kGemmMaxK = 32768;

// Launch the tcgen05 GEMM (error code, 0 on success).
int gemm_i8x4(const GemmJob& job, cudaStream_t stream);

// Bytes of the K-split partial-sum buffer the job needs (0: no split).
size_t gemm_partial_bytes(uint32_t rows, uint32_t cols, uint32_t Kp, uint32_t batch);

// Split an int16 matrix into the hi / lo planes row by row:
//   dst (b, r, kk) <- src[b*src_bs + r*ld + kk]   (kk < K, zero up to Kp)
int split_planes(const int16_t* src, uint64_t src_bs, uint32_t planes, uint32_t rows, uint64_t ld, uint32_t K,
                 uint32_t Kp, int8_t* hi, uint8_t* lo, cudaStream_t stream);

// Two such splits (A and B of one job) in a single launch.
struct SplitSeg {
  const int16_t* src;
  uint64_t src_bs;
  uint32_t planes, rows;
  uint64_t ld;
  uint32_t K, Kp;
  int8_t* hi;
  uint8_t* lo;
};
int split_planes2(const SplitSeg& a, const SplitSeg& b, cudaStream_t stream);

// Per-device word the kernels' bounded waits write on a timeout.
int* device_error_word();

// Read (after the work on `stream` — nullptr: the legacy default stream — has
// finished) and clear the status word of the allocation-free MatMul jobs on
// the current device; no allocation.
int noalloc_status_take(int* code, cudaStream_t stream);

}  // namespace corm
