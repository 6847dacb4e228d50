// MatmulKernel jobs on sm_100a.  Register semantics: phoenix367/cormorant
// inference-scheduler/test/host_emu.py:312-362 (kernels/matmul_rtl/model/
// include/MatmulKernel.h:195-242): per batch slice C[r][j] = sat16(floor(
// sum_kk A[r][kk] B[kk][j] / 2^8)) with B row-major, packed tile-major or in
// the GEMV image; the simulator's Q8.8 path (inference-scheduler/src/codegen/
// _simulate.py:620-633) is the exact sum, its exponent path (:814-835) the
// int32-wrapped one (CORM_F_WRAP32).
//
// n >= 3 rows: the operands are split into int8 planes (A K-major, B as it
// lies, MN-major) and multiplied on the tensor cores (gemm_i8x4.cu); the TMA
// fills the rows of a 128-row tile beyond n with zeros.
// n <= 2 rows (GEMV, HBM-bound on B): a CUDA-core kernel reads int16 B once
// with 16-byte loads, 8 columns x n rows of int64 sums per lane, splitting K
// across CTAs (exact integer atomics) when the output alone is too small to
// fill the GPU.
#include <mutex>

#include "corm_common.cuh"
#include "gemm_i8x4.h"

namespace {

constexpr uint32_t kTileM = 32;      // packed-B tile width (platforms/kv260.json kernels.matmul.tile_m)
constexpr uint32_t kMaxK = 4096;     // platforms/kv260.json kernels.matmul.max_k
constexpr uint32_t kSmallRows = 2;  // n at or below: CUDA-core path (above: tensor cores, M padded by TMA zero fill)

// offset of B[kk][j] (MatmulKernel.h matmul_packed_index / matmul_gemv_index)
__device__ __forceinline__ uint64_t b_offset(uint32_t kk, uint32_t j, uint32_t k, uint32_t m, uint32_t packed,
                                             uint32_t kw) {
  if (kw > 1) {
    const uint64_t c = (uint64_t)(kk / (16u * kw)) * 16u + kk % 16u;
    return (c * m + j) * kw + (kk / 16u) % kw;
  }
  if (packed) return ((uint64_t)(j / kTileM) * k + kk) * kTileM + j % kTileM;
  return (uint64_t)kk * m + j;
}

struct MmArgs {
  const int16_t* a;
  const int16_t* b;
  int16_t* c;
  uint32_t n, k, m, batch, a_bs, b_bs, c_bs, packed, kw, flags;
  corm::PostOp post;
};

__device__ __forceinline__ int16_t mm_finish(int64_t acc, uint32_t flags) {
  if (flags & CORM_F_WRAP32) acc = corm_wrap32(acc);
  int64_t y = corm_sat16(acc >> 8);
  if (flags & (CORM_F_ACT_RELU | CORM_F_ACT_RELU6)) y = y < 0 ? 0 : y;
  if ((flags & CORM_F_ACT_RELU6) && y > 1536) y = 1536;
  return (int16_t)y;
}

// B of any layout -> MN-major hi / lo planes [plane][k][Np]: 16 consecutive
// columns of one K row per thread (row-major B goes through split_planes).
__global__ void __launch_bounds__(256) split_b_gather_kernel(MmArgs p, uint32_t planes, uint32_t Np, int8_t* hi,
                                                             uint8_t* lo) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t per_row = Np / 16, total = (uint64_t)planes * p.k * per_row;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t row = i / per_row;  // plane * k + kk
    const uint32_t j0 = (uint32_t)(i - row * per_row) * 16;
    const uint32_t pl = (uint32_t)(row / p.k), kk = (uint32_t)(row % p.k);
    const int16_t* B = p.b + (uint64_t)pl * p.b_bs;
    uint32_t h[4], l[4];
#pragma unroll
    for (int w = 0; w < 4; w++) {
      h[w] = l[w] = 0;
#pragma unroll
      for (int e = 0; e < 4; e++) {
        const uint32_t j = j0 + 4 * w + e;
        const int16_t v = j < p.m ? __ldg(B + b_offset(kk, j, p.k, p.m, p.packed, p.kw)) : (int16_t)0;
        h[w] |= (uint32_t)(uint8_t)(v >> 8) << (8 * e);
        l[w] |= (uint32_t)(uint8_t)(v & 0xFF) << (8 * e);
      }
    }
    *(int4*)(hi + row * Np + j0) = make_int4((int)h[0], (int)h[1], (int)h[2], (int)h[3]);
    *(int4*)(lo + row * Np + j0) = make_int4((int)l[0], (int)l[1], (int)l[2], (int)l[3]);
  }
}

// GEMV path (n <= 2, HBM-bound on B): a warp owns 256 consecutive columns —
// 8 per lane, one 16-byte load per B row — over a K range, A values read as
// warp-wide broadcasts, int64 sums; the K range is split across CTAs when the
// grid alone would not fill the GPU, each range's sums stored in its own
// int64 slot (no memset, no atomics) and added by mm_small_finish.
template <int NR>
__global__ void __launch_bounds__(128) mm_gemv_kernel(MmArgs p, uint32_t kchunk, unsigned long long* partial) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const uint32_t j0 = (blockIdx.x * 4 + w) * 256 + lane * 8;
  const uint32_t bt = blockIdx.y;
  const uint32_t k_lo = blockIdx.z * kchunk, k_hi = min(p.k, k_lo + kchunk);
  const int16_t* A = p.a + (uint64_t)bt * p.a_bs;
  const int16_t* B = p.b + (uint64_t)bt * p.b_bs;
  if (j0 >= p.m) return;
  int64_t acc[NR][8];
#pragma unroll
  for (int r = 0; r < NR; r++)
#pragma unroll
    for (int e = 0; e < 8; e++) acc[r][e] = 0;
  const bool vec = p.kw <= 1 && !p.packed && (p.m % 8 == 0) && (((uintptr_t)B & 15) == 0) && j0 + 8 <= p.m;
  if (vec) {
#pragma unroll 4
    for (uint32_t kk = k_lo; kk < k_hi; kk++) {
      alignas(16) int16_t bv[8];
      *(int4*)bv = __ldg((const int4*)(B + (uint64_t)kk * p.m + j0));
#pragma unroll
      for (int r = 0; r < NR; r++) {
        const int32_t a = __ldg(A + (uint64_t)r * p.k + kk);
#pragma unroll
        for (int e = 0; e < 8; e++) acc[r][e] += (int64_t)(a * (int32_t)bv[e]);  // |a b| <= 2^30
      }
    }
  } else {
    for (uint32_t kk = k_lo; kk < k_hi; kk++) {
      int32_t bv[8];
#pragma unroll
      for (int e = 0; e < 8; e++)
        bv[e] = (j0 + e < p.m) ? __ldg(B + b_offset(kk, j0 + e, p.k, p.m, p.packed, p.kw)) : 0;
#pragma unroll
      for (int r = 0; r < NR; r++) {
        const int32_t a = __ldg(A + (uint64_t)r * p.k + kk);
#pragma unroll
        for (int e = 0; e < 8; e++) acc[r][e] += (int64_t)(a * bv[e]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < NR; r++) {
    if (r >= (int)p.n) continue;
#pragma unroll
    for (int e = 0; e < 8; e++) {
      const uint32_t jj = j0 + e;
      if (jj >= p.m) continue;
      if (partial) {  // this K range's slot: every (slot, batch, row, column) written once
        partial[(((uint64_t)blockIdx.z * p.batch + bt) * p.n + r) * p.m + jj] = (unsigned long long)acc[r][e];
      } else {
        const uint64_t off = (uint64_t)bt * p.c_bs + (uint64_t)r * p.m + jj;
        int16_t y = mm_finish(acc[r][e], p.flags);
        if (p.post.op != corm::kPostNone) y = corm::post_apply(p.post, y, corm::post_b(p.post, off, jj));
        p.c[off] = y;
      }
    }
  }
}

// the K ranges' int64 sums added (exact integer addition, so in any order):
// a warp per output, its lanes taking every 32nd range (up to 128 ranges
// would otherwise be a long chain of loads for one thread)
__global__ void mm_small_finish(MmArgs p, const unsigned long long* partial, uint32_t ks) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t total = (uint64_t)p.batch * p.n * p.m;
  const uint32_t lane = threadIdx.x & 31u;
  const uint64_t nwarps = ((uint64_t)gridDim.x * blockDim.x) >> 5;
  for (uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < total; i += nwarps) {
    unsigned long long acc = 0;
    for (uint32_t z = lane; z < ks; z += 32u) acc += __ldg(partial + z * total + i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane != 0) continue;
    const uint64_t bt = i / ((uint64_t)p.n * p.m), rem = i - bt * p.n * p.m;
    const uint64_t off = bt * p.c_bs + rem;
    int16_t y = mm_finish((int64_t)acc, p.flags);
    if (p.post.op != corm::kPostNone) y = corm::post_apply(p.post, y, corm::post_b(p.post, off, (uint32_t)(rem % p.m)));
    p.c[off] = y;
  }
}

struct Plan {
  bool small;
  uint32_t Kp, Np, a_planes, b_planes, ksplit, kchunk;
  size_t a_plane_bytes, b_plane_bytes, partial_bytes, bytes;
};

Plan plan_of(const corm_matmul_desc* d) {
  Plan pl{};
  pl.small = d->n <= kSmallRows;
  if (pl.small) {
    // enough CTAs for several waves: split K down to chunks of 16 rows (a
    // warp's serial chain of loads is then short)
    const uint64_t blocks = (uint64_t)((d->m + 1023) / 1024) * d->batch;
    uint32_t ks = 1;
    while (blocks * ks < 8 * 148 && d->k / (ks * 2) >= 16) ks *= 2;
    pl.kchunk = (d->k + ks - 1) / ks;
    pl.ksplit = (d->k + pl.kchunk - 1) / pl.kchunk;
    ks = pl.ksplit;
    pl.bytes = ks > 1 ? (size_t)ks * d->batch * d->n * d->m * 8 : 0;  // a slot per K range
    return pl;
  }
  pl.Kp = (d->k + 15u) / 16u * 16u;
  pl.Np = (d->m + 15u) / 16u * 16u;
  pl.a_planes = (d->a_batch_stride == 0 || d->batch == 1) ? 1 : d->batch;
  pl.b_planes = (d->b_batch_stride == 0 || d->batch == 1) ? 1 : d->batch;
  pl.a_plane_bytes = ((size_t)pl.a_planes * d->n * pl.Kp + 255) & ~(size_t)255;
  pl.b_plane_bytes = ((size_t)pl.b_planes * d->k * pl.Np + 255) & ~(size_t)255;  // MN-major [k][Np]
  pl.partial_bytes = corm::gemm_partial_bytes(d->n, d->m, pl.Kp, d->batch);
  pl.bytes = 2 * pl.a_plane_bytes + 2 * pl.b_plane_bytes + pl.partial_bytes;
  return pl;
}

// The tensor-core path of a job with n >= 3 rows.  Row-major B with K and m
// multiples of 8 on 16-byte aligned rows, and 1/n + 1/m above 1/500: the
// GEMM reads the int16 operands and splits them itself (only a K-split
// partial-sum buffer in the workspace); otherwise the operands are split into
// int8 planes first.  The workspace is sized for the second case.
int tensor_path(const corm_matmul_desc* d, const MmArgs& p, const Plan& pl, uint8_t* w, const corm::PostOp& post,
                int* err, cudaStream_t st, const corm_out_groups* grp = nullptr) {
  // The producer warps sustain fewer bytes in flight than the TMA: for large
  // tiles of work per operand byte (n and m both above ~1000) the split planes
  // plus TMA are faster, below it the saved split traffic wins.
  const bool direct = !d->b_packed && d->gemv_kw <= 1 && d->k % 8 == 0 && d->m % 8 == 0 &&
                      !(((uintptr_t)d->a | (uintptr_t)d->b) & 15u) &&
                      (d->batch == 1 || (d->a_batch_stride % 8 == 0 && d->b_batch_stride % 8 == 0)) &&
                      ((uint64_t)d->n + d->m) * 500u > (uint64_t)d->n * d->m;
  corm::GemmJob j{};
  j.rows = d->n;
  j.cols = d->m;
  j.Kp = pl.Kp;
  if (grp && grp->mulact) {  // gate / up pairs: one output of m / 2 columns
    j.mulact = 1;
    j.ma_sa = grp->ma_sa;
    j.ma_sc = grp->ma_sc;
  } else if (grp) {
    j.ngroups = grp->count;
    for (uint32_t g = 0; g < 4 && g < grp->count; g++) {
      j.gout[g] = grp->out[g];
      j.gw[g] = grp->width[g];
    }
  }
  j.batch = d->batch;
  j.a_planes = pl.a_planes;
  j.b_planes = pl.b_planes;
  j.b_mn = 1;
  j.K = d->k;
  j.cols_p = pl.Np;
  j.mode = 0;
  j.out = d->c;
  j.out_batch_stride = d->c_batch_stride;
  j.ldc = j.mulact ? d->m / 2 : d->m;
  j.flags = d->flags;
  j.post = post;
  j.err = err;
  if (direct) {
    j.a16 = d->a;
    j.b16 = d->b;
    j.a_bs16 = pl.a_planes == 1 ? 0 : d->a_batch_stride;
    j.b_bs16 = pl.b_planes == 1 ? 0 : d->b_batch_stride;
    j.lda = d->k;
    j.ldb = d->m;
    j.partial = pl.partial_bytes ? (void*)w : nullptr;
    return corm::gemm_i8x4(j, st);
  }
  int8_t* a_hi = (int8_t*)w;
  uint8_t* a_lo = w + pl.a_plane_bytes;
  int8_t* b_hi = (int8_t*)(w + 2 * pl.a_plane_bytes);
  uint8_t* b_lo = w + 2 * pl.a_plane_bytes + pl.b_plane_bytes;
  if (!d->b_packed && d->gemv_kw <= 1) {
    // row-major B is already MN-major: both operands split elementwise in one
    // launch (B rows of m padded to Np)
    const corm::SplitSeg sa{d->a, d->a_batch_stride, pl.a_planes, d->n, d->k, d->k, pl.Kp, a_hi, a_lo};
    const corm::SplitSeg sb{d->b, d->b_batch_stride, pl.b_planes, d->k, d->m, d->m, pl.Np, b_hi, b_lo};
    if (int rc = corm::split_planes2(sa, sb, st)) return rc;
  } else {
    if (int rc = corm::split_planes(d->a, d->a_batch_stride, pl.a_planes, d->n, d->k, d->k, pl.Kp, a_hi, a_lo, st))
      return rc;
    const uint64_t total = (uint64_t)pl.b_planes * d->k * (pl.Np / 16);
    {
      corm::ProfScope prof_("split_b_gather_kernel", st);
      corm_launch_pdl(split_b_gather_kernel, dim3(corm_blocks(total, 256, 148u * 16u)), dim3(256), 0, st, p, pl.b_planes, pl.Np, b_hi, b_lo);
    }
    if (int rc = corm::cuda_status("matmul split_b")) return rc;
  }
  j.a_hi = a_hi;
  j.a_lo = a_lo;
  j.b_hi = b_hi;
  j.b_lo = b_lo;
  j.partial = pl.partial_bytes ? (void*)(w + 2 * pl.a_plane_bytes + 2 * pl.b_plane_bytes) : nullptr;
  return corm::gemm_i8x4(j, st);
}

int validate(const corm_matmul_desc* d) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_matmul: null descriptor");
  if (d->k > kMaxK) return corm::fail(CORM_EINVAL, "corm_matmul: k %u beyond max_k %u", d->k, kMaxK);
  if (d->b_packed && d->gemv_kw) return corm::fail(CORM_EINVAL, "corm_matmul: b_packed with gemv_kw");
  if (d->gemv_kw && d->gemv_kw != 1 && d->gemv_kw != 2 && d->gemv_kw != 4 && d->gemv_kw != 8)
    return corm::fail(CORM_EINVAL, "corm_matmul: gemv_kw %u", d->gemv_kw);
  return CORM_OK;
}

}  // namespace

extern "C" int corm_matmul_workspace_size(const corm_matmul_desc* d, size_t* bytes) {
  if (int rc = validate(d)) return rc;
  if (!bytes) return corm::fail(CORM_EINVAL, "corm_matmul_workspace_size: null output");
  *bytes = (d->n && d->m && d->k && d->batch) ? plan_of(d).bytes : 0;
  return CORM_OK;
}

namespace {
int matmul_impl(const corm_matmul_desc* d, const corm::PostOp& post, cudaStream_t st);
}

extern "C" int corm_matmul(const corm_matmul_desc* d, corm_stream_t stream) {
  return matmul_impl(d, corm::PostOp{}, (cudaStream_t)stream);
}

extern "C" int corm_matmul_post(const corm_matmul_desc* d, const corm_postop* post, corm_stream_t stream) {
  corm::PostOp q;
  if (int rc = corm::make_postop(post, q)) return rc;
  return matmul_impl(d, q, (cudaStream_t)stream);
}

namespace {
// k = 0: every output is floor(0) = 0.  Each batch's n x m run is cleared, in
// one call for all of them.
int clear_outputs(const corm_matmul_desc* d, cudaStream_t st, const char* who) {
  const size_t run = (size_t)d->n * d->m * 2;
  cudaError_t e;
  if (d->batch == 1)
    e = cudaMemsetAsync(d->c, 0, run, st);
  else if ((size_t)d->c_batch_stride * 2 >= run)
    e = cudaMemset2DAsync(d->c, (size_t)d->c_batch_stride * 2, 0, run, d->batch, st);
  else  // batches that share rows: clear from the first output to the last
    e = cudaMemsetAsync(d->c, 0, (size_t)(d->batch - 1) * d->c_batch_stride * 2 + run, st);
  if (e != cudaSuccess) return corm::cuda_status(who);
  return CORM_OK;
}

int matmul_impl(const corm_matmul_desc* d, const corm::PostOp& post, cudaStream_t st) {
  if (int rc = validate(d)) return rc;
  if (int rc = corm::check_device()) return rc;
  if (d->n == 0 || d->m == 0 || d->batch == 0) return CORM_OK;
  if (!d->a || !d->b || !d->c) return corm::fail(CORM_EINVAL, "corm_matmul: null operand");
  if (post.op != corm::kPostNone && d->k == 0)
    return corm::fail(CORM_EINVAL, "corm_matmul_post: k = 0");
  MmArgs p{d->a, d->b, d->c, d->n, d->k, d->m, d->batch, d->a_batch_stride, d->b_batch_stride, d->c_batch_stride,
           d->b_packed, d->gemv_kw, d->flags, post};
  if (d->k == 0) return clear_outputs(d, st, "corm_matmul");  // empty sum: floor(0) = 0 everywhere
  const Plan pl = plan_of(d);
  void* ws = d->workspace;
  if (pl.bytes) {
    if (ws && d->workspace_bytes < pl.bytes)
      return corm::fail(CORM_ENOMEM, "corm_matmul: workspace %zu < %zu bytes", d->workspace_bytes, pl.bytes);
    if (!ws && !(ws = corm::scratch(pl.bytes, st))) return CORM_ENOMEM;
  }
  if (pl.small) {
    unsigned long long* partial = pl.ksplit > 1 ? (unsigned long long*)ws : nullptr;
    dim3 grid((d->m + 1023) / 1024, d->batch, pl.ksplit);
    if (d->n <= 1) {
      corm::ProfScope prof_("mm_gemv_kernel<1>", st);
      corm_launch_pdl(mm_gemv_kernel<1>, grid, dim3(128), 0, st, p, pl.kchunk, partial);
    } else {  // n <= kSmallRows
      corm::ProfScope prof_("mm_gemv_kernel<2>", st);
      corm_launch_pdl(mm_gemv_kernel<2>, grid, dim3(128), 0, st, p, pl.kchunk, partial);
    }
    if (int rc = corm::cuda_status("matmul small")) return rc;
    if (partial) {
      {
        corm::ProfScope prof_("mm_small_finish", st);
        corm_launch_pdl(mm_small_finish, dim3(corm_blocks((uint64_t)d->batch * d->n * d->m * 32u, 256)), dim3(256), 0,
                        st, p, (const unsigned long long*)partial, pl.ksplit);
      }
      return corm::cuda_status("matmul small finish");
    }
    return CORM_OK;
  }
  return tensor_path(d, p, pl, (uint8_t*)ws, post, nullptr, st);
}
}  // namespace

// ---------------------------------------------------------------- allocation-free variant
// corm_matmul_noalloc: the same MatMul job for callers that must not allocate
// device memory once they are running — a generated inference project whose
// buffers all come from a pool sized at start-up, or a host whose device
// memory belongs to another allocator — so they can neither pass a workspace
// of their own nor let the library grow its scratch with cudaMalloc.  Its
// scratch (the int8 split planes and the K-split partial sums) is the
// file-scope array below, which every GPU that loads this library holds until
// the process exits; jobs needing more than kNoAllocBytes are rejected.
namespace {

constexpr size_t kNoAllocBytes = 64ull << 20;  // 64 MiB per device
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];
static __device__ int g_noalloc_status;  // the GEMM's bounded waits report here

struct NoAllocDev {
  uint8_t* scratch = nullptr;
  int* status = nullptr;
};
NoAllocDev g_noalloc[64];
std::mutex g_noalloc_mu;

// Once per device, with that device current: the device addresses of the
// file-scope array and status word (host code only ever sees a stand-in for
// the symbol itself, never a device address).
int noalloc_setup(NoAllocDev& out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return corm::fail(CORM_ECUDA, "noalloc: no device");
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDev& s = g_noalloc[dev];
  if (!s.scratch) {
    void* p = nullptr;
    void* q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return corm::fail(CORM_ECUDA, "noalloc: cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&q, g_noalloc_status);
    if (e != cudaSuccess) return corm::fail(CORM_ECUDA, "noalloc: cudaGetSymbolAddress(status): %s", cudaGetErrorString(e));
    s.status = (int*)q;
    s.scratch = (uint8_t*)p;
  }
  out = s;
  return CORM_OK;
}

}  // namespace

namespace corm {
int noalloc_status_take(int* code, cudaStream_t st) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_noalloc_status, sizeof v, 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess && v) {
    static const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_noalloc_status, &zero, sizeof zero, 0, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  }
  if (e != cudaSuccess) return fail(CORM_ECUDA, "noalloc status: %s", cudaGetErrorString(e));
  if (code) *code = v;
  return CORM_OK;
}
}  // namespace corm

extern "C" int corm_matmul_noalloc_status(int* code, corm_stream_t stream) {
  if (int rc = corm::check_device()) return rc;
  return corm::noalloc_status_take(code, (cudaStream_t)stream);
}

extern "C" int corm_matmul_noalloc(const corm_matmul_desc* d, corm_stream_t stream) {
  if (int rc = validate(d)) return rc;
  if (int rc = corm::check_device()) return rc;
  if (d->n == 0 || d->m == 0 || d->batch == 0) return CORM_OK;
  if (!d->a || !d->b || !d->c) return corm::fail(CORM_EINVAL, "corm_matmul_noalloc: null operand");
  cudaStream_t st = (cudaStream_t)stream;
  MmArgs p{d->a, d->b, d->c, d->n, d->k, d->m, d->batch, d->a_batch_stride, d->b_batch_stride, d->c_batch_stride,
           d->b_packed, d->gemv_kw, d->flags};
  if (d->k == 0) return clear_outputs(d, st, "corm_matmul_noalloc");  // every output is 0
  const Plan pl = plan_of(d);
  if (pl.bytes > kNoAllocBytes)
    return corm::fail(CORM_ELIMIT, "corm_matmul_noalloc: the job needs %zu bytes of scratch, beyond the %zu-byte "
                      "static scratch (use corm_matmul with a workspace)", pl.bytes, kNoAllocBytes);
  NoAllocDev na;
  if (int rc = noalloc_setup(na)) return rc;
  uint8_t* w = na.scratch;
  if (pl.small) {
    unsigned long long* partial = pl.ksplit > 1 ? (unsigned long long*)w : nullptr;
    dim3 grid((d->m + 1023) / 1024, d->batch, pl.ksplit);
    if (d->n <= 1) {
      corm::ProfScope prof_("mm_gemv_kernel<1>", st);
      corm_launch_pdl(mm_gemv_kernel<1>, grid, dim3(128), 0, st, p, pl.kchunk, partial);
    } else {  // n <= kSmallRows
      corm::ProfScope prof_("mm_gemv_kernel<2>", st);
      corm_launch_pdl(mm_gemv_kernel<2>, grid, dim3(128), 0, st, p, pl.kchunk, partial);
    }
    if (int rc = corm::cuda_status("matmul_noalloc small")) return rc;
    if (partial) {
      {
        corm::ProfScope prof_("mm_small_finish", st);
        corm_launch_pdl(mm_small_finish, dim3(corm_blocks((uint64_t)d->batch * d->n * d->m * 32u, 256)), dim3(256), 0,
                        st, p, (const unsigned long long*)partial, pl.ksplit);
      }
      return corm::cuda_status("matmul_noalloc small finish");
    }
    return CORM_OK;
  }
  return tensor_path(d, p, pl, w, corm::PostOp{}, na.status, st);
}

// ---------------------------------------------------------------- column groups
// corm_matmul_groups: one MatMul job whose output columns go to several
// buffers — sibling projections (q / k / v, gate / up) over their concatenated
// weights in one launch.  The tensor-core path only (n > 2), no fused job.
extern "C" int corm_matmul_groups(const corm_matmul_desc* d, const corm_out_groups* g, corm_stream_t stream) {
  if (int rc = validate(d)) return rc;
  if (int rc = corm::check_device()) return rc;
  if (!g || g->count < 1 || g->count > 4) return corm::fail(CORM_EINVAL, "corm_matmul_groups: 1..4 output groups");
  if (!d->a || !d->b) return corm::fail(CORM_EINVAL, "corm_matmul_groups: null operand");
  if (d->n <= kSmallRows || d->k == 0)
    return corm::fail(CORM_EINVAL, "corm_matmul_groups: n %u / k %u (the tensor-core path: n > %u, k > 0)", d->n, d->k,
                      kSmallRows);
  if (d->n == 0 || d->m == 0 || d->batch == 0) return CORM_OK;
  if (g->mulact && (g->count != 1 || d->m % 32u || g->width[0] != d->m / 2 || !g->out[0]))
    return corm::fail(CORM_EINVAL, "corm_matmul_groups: gate / up pairs need one output of m / 2 columns, m %% 32 == 0");
  cudaStream_t st = (cudaStream_t)stream;
  corm_matmul_desc dd = *d;
  dd.c = g->out[0];
  dd.c_batch_stride = d->n * g->width[0];
  MmArgs p{dd.a, dd.b, dd.c, dd.n, dd.k, dd.m, dd.batch, dd.a_batch_stride, dd.b_batch_stride, dd.c_batch_stride,
           dd.b_packed, dd.gemv_kw, dd.flags, corm::PostOp{}};
  const Plan pl = plan_of(&dd);
  void* ws = d->workspace;
  if (pl.bytes) {
    if (ws && d->workspace_bytes < pl.bytes)
      return corm::fail(CORM_ENOMEM, "corm_matmul_groups: workspace %zu < %zu bytes", d->workspace_bytes, pl.bytes);
    if (!ws && !(ws = corm::scratch(pl.bytes, st))) return CORM_ENOMEM;
  }
  return tensor_path(&dd, p, pl, (uint8_t*)ws, corm::PostOp{}, nullptr, st, g);
}

// ---------------------------------------------------------------- constant weights split once
// corm_split_b_planes / corm_matmul_bplanes: a weight that many jobs read is
// split into its int8 hi / lo planes once; the GEMM then loads the planes by
// TMA and splits only A (into tensor memory) — for few rows, where splitting
// the weight inside every job is the GEMM's largest cost.
extern "C" int corm_split_b_planes(const int16_t* b, uint32_t k, uint32_t m, int8_t* hi, uint8_t* lo,
                                   corm_stream_t stream) {
  if (int rc = corm::check_device()) return rc;
  if (!b || !hi || !lo || k == 0 || m == 0) return corm::fail(CORM_EINVAL, "corm_split_b_planes: null buffer or empty");
  const uint32_t mp = (m + 15u) / 16u * 16u;
  return corm::split_planes(b, 0, 1, k, m, m, mp, hi, lo, (cudaStream_t)stream);
}

extern "C" int corm_matmul_bplanes(const corm_matmul_desc* d, const int8_t* b_hi, const uint8_t* b_lo,
                                   const corm_out_groups* g, corm_stream_t stream) {
  if (int rc = validate(d)) return rc;
  if (int rc = corm::check_device()) return rc;
  if (!d->a || !b_hi || !b_lo || (!g && !d->c)) return corm::fail(CORM_EINVAL, "corm_matmul_bplanes: null operand");
  if (g && (g->count < 1 || g->count > 4)) return corm::fail(CORM_EINVAL, "corm_matmul_bplanes: 1..4 output groups");
  if (d->n <= kSmallRows || d->k == 0 || d->k % 8u || ((uintptr_t)d->a & 15u) ||
      (d->batch > 1 && (d->a_batch_stride % 8u || d->b_batch_stride != 0)) || d->b_packed || d->gemv_kw > 1)
    return corm::fail(CORM_EINVAL,
                      "corm_matmul_bplanes: n %u, k %u (n > %u, k a multiple of 8, A on 16-byte rows, one B for "
                      "every batch, row-major)", d->n, d->k, kSmallRows);
  if (d->m == 0 || d->batch == 0) return CORM_OK;
  cudaStream_t st = (cudaStream_t)stream;
  corm::GemmJob j{};
  j.rows = d->n;
  j.cols = d->m;
  j.Kp = (d->k + 15u) / 16u * 16u;
  j.batch = d->batch;
  j.a_planes = d->batch;
  j.b_planes = 1;
  j.b_mn = 1;
  j.K = d->k;
  j.cols_p = (d->m + 15u) / 16u * 16u;
  j.mode = 0;
  j.out = g ? g->out[0] : d->c;
  j.out_batch_stride = d->c_batch_stride;
  j.ldc = d->m;
  j.flags = d->flags;
  j.a16 = d->a;
  j.a_bs16 = d->batch == 1 ? 0 : d->a_batch_stride;
  j.lda = d->k;
  j.b_hi = b_hi;
  j.b_lo = b_lo;
  if (g && g->mulact) {  // gate / up pairs: one output of m / 2 columns
    if (g->count != 1 || d->m % 32u || g->width[0] != d->m / 2 || !g->out[0])
      return corm::fail(CORM_EINVAL, "corm_matmul_bplanes: gate / up pairs need one output of m / 2 columns");
    j.mulact = 1;
    j.ma_sa = g->ma_sa;
    j.ma_sc = g->ma_sc;
    j.ldc = d->m / 2;
    j.out_batch_stride = (uint64_t)d->n * (d->m / 2);
  } else if (g) {
    j.ngroups = g->count;
    for (uint32_t q = 0; q < g->count; q++) {
      j.gout[q] = g->out[q];
      j.gw[q] = g->width[q];
    }
  }
  const size_t pb = corm::gemm_partial_bytes(j.rows, j.cols, j.Kp, j.batch);
  if (pb) {
    void* ws = d->workspace;
    if (ws && d->workspace_bytes < pb)
      return corm::fail(CORM_ENOMEM, "corm_matmul_bplanes: workspace %zu < %zu bytes", d->workspace_bytes, pb);
    if (!ws && !(ws = corm::scratch(pb, st))) return CORM_ENOMEM;
    j.partial = ws;
  }
  return corm::gemm_i8x4(j, st);
}
