// tcgen05 kind::i8 GEMM with the four-way int16 split (see gemm_i8x4.h).
//
// CTA = 6 warps, one 128 x 128 output tile, warp-specialised:
//   warp 0      TMA producer: per 128-byte K block, 4 tiles (A hi/lo, B hi/lo,
//               128 rows x 128 bytes each, 128-byte swizzle) into a STAGES-deep ring
//   warp 1      TMEM owner (512 columns) and MMA issuer: 16 tcgen05.mma
//               (128x128x32) per K block into HH / MID / LL, commit frees the slot
//   warps 2..5  epilogue: tcgen05.ld of the three accumulators, int64 recombine,
//               the job's rounding rule, int16 stores
// Every mbarrier wait is bounded (sm100::mbar_wait); a timeout leaves an error
// code in the per-device error word and the CTA unwinds (TMEM freed).
#include <cudaTypedefs.h>

#include <mutex>

#include "corm_common.cuh"
#include "corm_sm100.cuh"
#include "gemm_i8x4.h"

namespace corm {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;  // BK in bytes = int8 elements
constexpr int STAGES = 3;
constexpr int TILE_BYTES = BM * BK;  // 16 KB (BM == BN)
constexpr int STAGE_BYTES = 4 * TILE_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t TMEM_COLS = 512;
constexpr int THREADS = 192;

struct EpiArgs {
  int mode;
  int16_t* out;
  uint64_t out_batch_stride;
  uint32_t ldc, rows, cols;
  uint32_t P, y_cn, y_cs, y_gs;
  uint64_t img_stride;
  const int16_t* bias;
  uint32_t flags;
  uint32_t num_kb, a_planes, b_planes;
  int* err;
};

__device__ __forceinline__ int16_t finish(int64_t acc, uint32_t flags) {
  if (flags & CORM_F_WRAP32) acc = corm_wrap32(acc);
  int64_t y = corm_sat16(acc >> 8);
  if (flags & (CORM_F_ACT_RELU | CORM_F_ACT_RELU6)) y = y < 0 ? 0 : y;
  if ((flags & CORM_F_ACT_RELU6) && y > 1536) y = 1536;
  return (int16_t)y;
}

__global__ void __launch_bounds__(THREADS, 1)
    gemm_i8x4_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                     const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                     const EpiArgs ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint32_t* tmem_slot = (uint32_t*)(tmem_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t tile_r = blockIdx.x * BM, tile_c = blockIdx.y * BN, bz = blockIdx.z;
  const int a_z = ep.a_planes == 1 ? 0 : (int)bz, b_z = ep.b_planes == 1 ? 0 : (int)bz;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      sm100::mbar_init(&full[s], 1);
      sm100::mbar_init(&empty[s], 1);
    }
    sm100::mbar_init(tmem_full, 1);
    sm100::fence_mbar_init();
  }
  if (warp == 1) sm100::tmem_alloc<TMEM_COLS>(tmem_slot);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    sm100::prefetch_tmap(&map_ahi);
    sm100::prefetch_tmap(&map_alo);
    sm100::prefetch_tmap(&map_bhi);
    sm100::prefetch_tmap(&map_blo);
    uint32_t issued = 0;
    bool ok = true;
    for (uint32_t kb = 0; kb < ep.num_kb; kb++) {
      const int s = kb % STAGES;
      if (kb >= (uint32_t)STAGES && !sm100::mbar_wait(&empty[s], ((kb / STAGES) - 1) & 1, ep.err, 101)) {
        ok = false;
        break;
      }
      uint8_t* st = smem + s * STAGE_BYTES;
      sm100::mbar_expect_tx(&full[s], STAGE_BYTES);
      const int x = (int)(kb * BK);
      sm100::tma_load_3d(st, &map_ahi, &full[s], x, (int)tile_r, a_z);
      sm100::tma_load_3d(st + TILE_BYTES, &map_alo, &full[s], x, (int)tile_r, a_z);
      sm100::tma_load_3d(st + 2 * TILE_BYTES, &map_bhi, &full[s], x, (int)tile_c, b_z);
      sm100::tma_load_3d(st + 3 * TILE_BYTES, &map_blo, &full[s], x, (int)tile_c, b_z);
      issued++;
    }
    if (!ok) {
      // let the loads already issued land before the CTA's shared memory goes away
      const uint32_t first = issued > (uint32_t)STAGES ? issued - STAGES : 0;
      for (uint32_t kb = first; kb < issued; kb++) {
        sm100::mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1, nullptr, 0, 200000000ll);
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t ID_SS = sm100::idesc_i8(BM, BN, 1, 1);
    constexpr uint32_t ID_SU = sm100::idesc_i8(BM, BN, 1, 0);
    constexpr uint32_t ID_US = sm100::idesc_i8(BM, BN, 0, 1);
    constexpr uint32_t ID_UU = sm100::idesc_i8(BM, BN, 0, 0);
    const uint32_t acc_hh = tmem, acc_mid = tmem + BN, acc_ll = tmem + 2 * BN;
    for (uint32_t kb = 0; kb < ep.num_kb; kb++) {
      const int s = kb % STAGES;
      if (!sm100::mbar_wait(&full[s], (kb / STAGES) & 1, ep.err, 102)) break;
      sm100::tc_fence_after();
      const uint32_t base = sm100::smem_u32(smem + s * STAGE_BYTES);
      const uint64_t d_ahi = sm100::sdesc_sw128(base), d_alo = sm100::sdesc_sw128(base + TILE_BYTES);
      const uint64_t d_bhi = sm100::sdesc_sw128(base + 2 * TILE_BYTES), d_blo = sm100::sdesc_sw128(base + 3 * TILE_BYTES);
#pragma unroll
      for (int ks = 0; ks < BK / 32; ks++) {
        const uint64_t adv = (uint64_t)((ks * 32) >> 4);  // 32-byte K step inside the swizzled row
        const uint32_t acc = (kb | ks) ? 1u : 0u;
        sm100::mma_i8(acc_hh, d_ahi + adv, d_bhi + adv, ID_SS, acc);
        sm100::mma_i8(acc_mid, d_ahi + adv, d_blo + adv, ID_SU, acc);
        sm100::mma_i8(acc_mid, d_alo + adv, d_bhi + adv, ID_US, 1u);
        sm100::mma_i8(acc_ll, d_alo + adv, d_blo + adv, ID_UU, acc);
      }
      sm100::mma_commit(&empty[s]);
    }
    sm100::mma_commit(tmem_full);  // also on failure: completes once every issued MMA has
  } else if (warp >= 2) {
    // ---------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool ok = sm100::mbar_wait(tmem_full, 0, ep.err, 103) && *(volatile int*)ep.err == 0;
    sm100::tc_fence_after();
    const uint32_t r = tile_r + q * 32 + lane;
    // row addressing
    uint64_t row_off = 0;
    if (ep.mode == 0) {
      row_off = (uint64_t)bz * ep.out_batch_stride + (uint64_t)r * ep.ldc;
    } else if (r < ep.rows) {
      const uint32_t n = r / ep.P, p = r - n * ep.P;
      row_off = (uint64_t)n * ep.img_stride + p;
    }
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    for (int cc = 0; cc < BN; cc += 32) {
      uint32_t hh[32], mid[32], ll[32];
      sm100::tmem_ld32(tmem + lane_addr + cc, hh);
      sm100::tmem_ld32(tmem + lane_addr + BN + cc, mid);
      sm100::tmem_ld32(tmem + lane_addr + 2 * BN + cc, ll);
      sm100::tmem_ld_wait();
      if (!ok || r >= ep.rows) continue;
      const uint32_t c0 = tile_c + cc;
      if (ep.mode == 0) {
        int16_t* dst = ep.out + row_off + c0;
        alignas(16) int16_t v[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int64_t acc = ((int64_t)(int32_t)hh[j] << 16) + ((int64_t)(int32_t)mid[j] << 8) + (int64_t)(int32_t)ll[j];
          v[j] = finish(acc, ep.flags);
        }
        if (c0 + 32 <= ep.cols && ((uintptr_t)dst & 15) == 0) {
#pragma unroll
          for (int j = 0; j < 4; j++) ((int4*)dst)[j] = ((const int4*)v)[j];
        } else {
#pragma unroll
          for (int j = 0; j < 32; j++)
            if (c0 + j < ep.cols) dst[j] = v[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const uint32_t c = c0 + j;
          if (c >= ep.cols) continue;
          int64_t acc = ((int64_t)(int32_t)hh[j] << 16) + ((int64_t)(int32_t)mid[j] << 8) + (int64_t)(int32_t)ll[j];
          if (ep.bias) acc += (int64_t)ep.bias[c] << 8;
          const uint64_t coff = ep.y_cn ? (uint64_t)(c % ep.y_cn) * ep.y_cs + (uint64_t)(c / ep.y_cn) * ep.y_gs
                                        : (uint64_t)c * ep.y_cs;
          ep.out[row_off + coff] = finish(acc, ep.flags);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc<TMEM_COLS>(tmem);
  }
}

// ---------------------------------------------------------------- split kernel
// dst (b, r, kk) <- src[b*bs + r*ld + kk]; 16 consecutive kk per thread, two
// 16-byte loads when the row is 16-byte aligned, 16-byte stores to each plane.
__global__ void __launch_bounds__(256) split_rows_kernel(const int16_t* __restrict__ src, uint64_t bs, uint32_t rows,
                                                         uint64_t ld, uint32_t K, uint32_t Kp, uint64_t total16,
                                                         int8_t* __restrict__ hi, uint8_t* __restrict__ lo) {
  const uint32_t per_row = Kp / 16;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total16; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = i / per_row;  // b * rows + r
    const uint32_t k0 = (uint32_t)(i - row * per_row) * 16;
    const uint64_t b = row / rows, r = row - b * rows;
    const int16_t* s = src + b * bs + r * ld + k0;
    alignas(16) int16_t v[16];
    if (k0 + 16 <= K && ((uintptr_t)s & 15) == 0) {
      *(int4*)v = __ldg((const int4*)s);
      *(int4*)(v + 8) = __ldg((const int4*)(s + 8));
    } else {
#pragma unroll
      for (int j = 0; j < 16; j++) v[j] = (k0 + j < K) ? __ldg(s + j) : (int16_t)0;
    }
    uint32_t h[4], l[4];
#pragma unroll
    for (int w = 0; w < 4; w++) {
      h[w] = l[w] = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        h[w] |= (uint32_t)(uint8_t)(v[4 * w + e] >> 8) << (8 * e);
        l[w] |= (uint32_t)(uint8_t)(v[4 * w + e] & 0xFF) << (8 * e);
      }
    }
    *(int4*)(hi + row * Kp + k0) = make_int4((int)h[0], (int)h[1], (int)h[2], (int)h[3]);
    *(int4*)(lo + row * Kp + k0) = make_int4((int)l[0], (int)l[1], (int)l[2], (int)l[3]);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// [planes][rows][Kp] bytes, box 128 (K) x 128 (rows) x 1, 128-byte swizzle
bool make_map(CUtensorMap* map, const void* base, uint32_t Kp, uint32_t rows, uint32_t planes) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {Kp, rows, planes};
  cuuint64_t strides[2] = {Kp, (cuuint64_t)Kp * rows};
  cuuint32_t box[3] = {BK, BM, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int* g_err_word[64];
std::mutex g_err_mu;

}  // namespace

int* device_error_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(g_err_mu);
  if (!g_err_word[dev]) {
    void* p = nullptr;
    if (cudaMalloc(&p, 256) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, 256);
    g_err_word[dev] = (int*)p;
  }
  return g_err_word[dev];
}

int split_planes(const int16_t* src, uint64_t src_bs, uint32_t planes, uint32_t rows, uint64_t ld, uint32_t K,
                 uint32_t Kp, int8_t* hi, uint8_t* lo, cudaStream_t stream) {
  const uint64_t total16 = (uint64_t)planes * rows * (Kp / 16);
  if (total16 == 0) return CORM_OK;
  {
    corm::ProfScope prof_("split_rows_kernel", stream);
    split_rows_kernel<<<corm_blocks(total16, 256, 148u * 16u), 256, 0, stream>>>(src, src_bs, rows, ld, K, Kp, total16, hi,
                                                                              lo);
  }
  return cuda_status("split_planes");
}

int gemm_i8x4(const GemmJob& j, cudaStream_t stream) {
  if (j.Kp % 16 || j.Kp == 0 || j.Kp > kGemmMaxK + 128)
    return fail(CORM_ELIMIT, "gemm: K %u outside 1..%u", j.Kp, kGemmMaxK);
  int* err = device_error_word();
  if (!err) return fail(CORM_ECUDA, "gemm: error word allocation failed");
  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  if (!make_map(&m_ahi, j.a_hi, j.Kp, j.rows, j.a_planes) || !make_map(&m_alo, j.a_lo, j.Kp, j.rows, j.a_planes) ||
      !make_map(&m_bhi, j.b_hi, j.Kp, j.cols, j.b_planes) || !make_map(&m_blo, j.b_lo, j.Kp, j.cols, j.b_planes))
    return fail(CORM_ECUDA, "gemm: cuTensorMapEncodeTiled failed");
  EpiArgs ep{};
  ep.mode = j.mode;
  ep.out = j.out;
  ep.out_batch_stride = j.out_batch_stride;
  ep.ldc = j.ldc;
  ep.rows = j.rows;
  ep.cols = j.cols;
  ep.P = j.P;
  ep.y_cn = j.y_cn;
  ep.y_cs = j.y_cs;
  ep.y_gs = j.y_gs;
  ep.img_stride = j.img_stride;
  ep.bias = j.bias;
  ep.flags = j.flags;
  ep.num_kb = (j.Kp + BK - 1) / BK;
  ep.a_planes = j.a_planes;
  ep.b_planes = j.b_planes;
  ep.err = err;
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaFuncSetAttribute(gemm_i8x4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set[dev] = true;
  }
  dim3 grid((j.rows + BM - 1) / BM, (j.cols + BN - 1) / BN, j.batch);
  if (grid.y > 65535 || grid.z > 65535) return fail(CORM_ELIMIT, "gemm: grid %u x %u x %u", grid.x, grid.y, grid.z);
  {
    corm::ProfScope prof_("gemm_i8x4_kernel", stream);
    gemm_i8x4_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(m_ahi, m_alo, m_bhi, m_blo, ep);
  }
  return cuda_status("gemm_i8x4");
}

}  // namespace corm

// Reads and clears the per-device word the kernels' bounded waits set on a
// timeout (synchronises the device first).  0 = no timeout since the last call.
extern "C" int corm_device_status(int* code) {
  int* w = corm::device_error_word();
  if (!w) return corm::fail(CORM_ECUDA, "corm_device_status: no error word");
  if (cudaDeviceSynchronize() != cudaSuccess) return corm::cuda_status("corm_device_status");
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return corm::cuda_status("corm_device_status");
  if (v) cudaMemset(w, 0, sizeof v);
  if (code) *code = v;
  return CORM_OK;
}
