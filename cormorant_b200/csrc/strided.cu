// Two jobs with no counterpart among the reference's kernel registers, used by
// the simulator to run the prefill attention of many sequences at once:
//
// corm_gemm_strided — the MatMul job's numerics (exact int16 sum, optional
// int32 wrap, floor / 2^8, sat16, optional ReLU / Clip) over a strided batch:
// row strides lda / ldb / ldc and batch strides per operand, B optionally
// given transposed ([m][k]).  One launch for the q.K^T or P.V of every
// sequence of a KV group (inference-scheduler/src/llm_nodes.py:1407-1423 per
// sequence).
//
// corm_copy_nd — an int16 copy between two strided views of up to six
// dimensions (the q image, the cache rows and the head merge of the
// attention: llm_nodes.py:1112-1143, 1645-1657).  A view whose innermost
// dimension differs between source and destination goes through 32 x 32
// shared-memory tiles, so both sides are read and written along their
// contiguous dimension.
#include "corm_common.cuh"
#include "gemm_i8x4.h"

namespace {

struct GsPlan {
  bool direct;
  uint32_t Kp, Np, a_planes, b_planes;
  size_t a_plane_bytes, b_plane_bytes, partial_bytes, bytes;
};

GsPlan gs_plan(const corm_gemm_desc* d) {
  GsPlan p{};
  p.Kp = (d->k + 15u) / 16u * 16u;
  p.Np = (d->m + 15u) / 16u * 16u;
  p.a_planes = (d->a_batch_stride == 0 || d->batch == 1) ? 1 : d->batch;
  p.b_planes = (d->b_batch_stride == 0 || d->batch == 1) ? 1 : d->batch;
  p.a_plane_bytes = ((size_t)p.a_planes * d->n * p.Kp + 255) & ~(size_t)255;
  p.b_plane_bytes = d->b_trans ? (((size_t)p.b_planes * d->m * p.Kp + 255) & ~(size_t)255)
                               : (((size_t)p.b_planes * d->k * p.Np + 255) & ~(size_t)255);
  p.partial_bytes = corm::gemm_partial_bytes(d->n, d->m, p.Kp, d->batch);
  p.bytes = 2 * p.a_plane_bytes + 2 * p.b_plane_bytes + p.partial_bytes;
  // int16 operands read by the GEMM's producer warps: 16-byte rows, MN-major B
  p.direct = !d->b_trans && d->k % 8 == 0 && d->m % 8 == 0 && d->lda % 8 == 0 && d->ldb % 8 == 0 &&
             !(((uintptr_t)d->a | (uintptr_t)d->b) & 15u) &&
             (p.a_planes == 1 || d->a_batch_stride % 8 == 0) && (p.b_planes == 1 || d->b_batch_stride % 8 == 0) &&
             ((uint64_t)d->n + d->m) * 500u > (uint64_t)d->n * d->m;
  return p;
}

int gs_validate(const corm_gemm_desc* d) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_gemm_strided: null descriptor");
  if (d->k > corm::kGemmMaxK) return corm::fail(CORM_ELIMIT, "corm_gemm_strided: k %u beyond %u", d->k, corm::kGemmMaxK);
  if (d->flags & ~(uint32_t)(CORM_F_WRAP32 | CORM_F_ACT_RELU | CORM_F_ACT_RELU6))
    return corm::fail(CORM_EINVAL, "corm_gemm_strided: flags 0x%x", d->flags);
  if (d->n && d->m && d->k) {
    if (d->lda < d->k || d->ldc < d->m || (d->b_trans ? d->ldb < d->k : d->ldb < d->m))
      return corm::fail(CORM_EINVAL, "corm_gemm_strided: a row stride below the row length");
  }
  return CORM_OK;
}

__global__ void gs_zero(corm_gemm_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t total = (uint64_t)d.batch * d.n * d.m;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t c = i % d.m, r = (i / d.m) % d.n, b = i / ((uint64_t)d.m * d.n);
    d.c[b * d.c_batch_stride + r * d.ldc + c] = 0;
  }
}

}  // namespace

extern "C" int corm_gemm_strided_workspace_size(const corm_gemm_desc* d, size_t* bytes) {
  if (int rc = gs_validate(d)) return rc;
  if (!bytes) return corm::fail(CORM_EINVAL, "corm_gemm_strided_workspace_size: null output");
  *bytes = (d->n && d->m && d->k && d->batch) ? gs_plan(d).bytes : 0;
  return CORM_OK;
}

extern "C" int corm_gemm_strided(const corm_gemm_desc* d, corm_stream_t stream) {
  if (int rc = gs_validate(d)) return rc;
  if (int rc = corm::check_device()) return rc;
  if (d->n == 0 || d->m == 0 || d->batch == 0) return CORM_OK;
  if (!d->a || !d->b || !d->c) return corm::fail(CORM_EINVAL, "corm_gemm_strided: null operand");
  cudaStream_t st = (cudaStream_t)stream;
  if (d->k == 0) {  // the empty sum: floor(0) = 0
    {
      corm::ProfScope prof_("gs_zero", st);
      corm_launch_pdl(gs_zero, dim3(corm_blocks((uint64_t)d->batch * d->n * d->m, 256)), dim3(256), 0, st, *d);
    }
    return corm::cuda_status("gemm_strided zero");
  }
  const GsPlan pl = gs_plan(d);
  uint8_t* w = (uint8_t*)d->workspace;
  if (pl.bytes) {
    if (w && d->workspace_bytes < pl.bytes)
      return corm::fail(CORM_ENOMEM, "corm_gemm_strided: workspace %zu < %zu bytes", d->workspace_bytes, pl.bytes);
    if (!w && !(w = (uint8_t*)corm::scratch(pl.bytes, st))) return CORM_ENOMEM;
  }
  corm::GemmJob j{};
  j.rows = d->n;
  j.cols = d->m;
  j.Kp = pl.Kp;
  j.batch = d->batch;
  j.a_planes = pl.a_planes;
  j.b_planes = pl.b_planes;
  j.K = d->k;
  j.cols_p = pl.Np;
  j.mode = 0;
  j.out = d->c;
  j.out_batch_stride = d->c_batch_stride;
  j.ldc = d->ldc;
  j.flags = d->flags;
  j.post = corm::PostOp{};
  if (pl.direct) {
    j.b_mn = 1;
    j.a16 = d->a;
    j.b16 = d->b;
    j.a_bs16 = pl.a_planes == 1 ? 0 : d->a_batch_stride;
    j.b_bs16 = pl.b_planes == 1 ? 0 : d->b_batch_stride;
    j.lda = d->lda;
    j.ldb = d->ldb;
    j.partial = pl.partial_bytes ? (void*)w : nullptr;
    return corm::gemm_i8x4(j, st);
  }
  int8_t* a_hi = (int8_t*)w;
  uint8_t* a_lo = w + pl.a_plane_bytes;
  int8_t* b_hi = (int8_t*)(w + 2 * pl.a_plane_bytes);
  uint8_t* b_lo = w + 2 * pl.a_plane_bytes + pl.b_plane_bytes;
  const corm::SplitSeg sa{d->a, pl.a_planes == 1 ? 0 : d->a_batch_stride, pl.a_planes, d->n, d->lda, d->k, pl.Kp,
                          a_hi, a_lo};
  // B as it lies: [k][m] rows split MN-major (rows of m padded to Np), or
  // transposed [m][k] rows split K-major
  const corm::SplitSeg sb = d->b_trans
      ? corm::SplitSeg{d->b, pl.b_planes == 1 ? 0 : d->b_batch_stride, pl.b_planes, d->m, d->ldb, d->k, pl.Kp, b_hi,
                       b_lo}
      : corm::SplitSeg{d->b, pl.b_planes == 1 ? 0 : d->b_batch_stride, pl.b_planes, d->k, d->ldb, d->m, pl.Np, b_hi,
                       b_lo};
  if (int rc = corm::split_planes2(sa, sb, st)) return rc;
  j.b_mn = d->b_trans ? 0 : 1;
  j.a_hi = a_hi;
  j.a_lo = a_lo;
  j.b_hi = b_hi;
  j.b_lo = b_lo;
  j.partial = pl.partial_bytes ? (void*)(w + 2 * pl.a_plane_bytes + 2 * pl.b_plane_bytes) : nullptr;
  return corm::gemm_i8x4(j, st);
}

// ---------------------------------------------------------------- corm_copy_nd
namespace {

constexpr int kMaxDims = 6;

struct CopyArgs {
  const int16_t* src;
  int16_t* dst;
  int nd;                     // dims after dropping size-1 ones (>= 1)
  uint32_t dims[kMaxDims];    // outermost first
  int64_t ss[kMaxDims], ds[kMaxDims];
  uint64_t total;
  // tiled path: the source's and the destination's unit-stride dims
  int is, id;
  uint64_t outer;             // elements / (dims[is] * dims[id])
};

// element i (row-major over dims) -> source and destination offsets
__device__ __forceinline__ void cp_offsets(const CopyArgs& a, uint64_t i, int64_t& so, int64_t& dof) {
  so = 0;
  dof = 0;
#pragma unroll
  for (int d = kMaxDims - 1; d >= 0; d--) {
    if (d < a.nd) {
      const uint64_t q = i / a.dims[d];
      const uint32_t x = (uint32_t)(i - q * a.dims[d]);
      so += (int64_t)x * a.ss[d];
      dof += (int64_t)x * a.ds[d];
      i = q;
    }
  }
}

__global__ void __launch_bounds__(256) copy_nd_elem(CopyArgs a) {
  corm_pdl_wait();
  corm_pdl_trigger();
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.total; i += (uint64_t)gridDim.x * blockDim.x) {
    int64_t so, dof;
    cp_offsets(a, i, so, dof);
    a.dst[dof] = a.src[so];
  }
}

// innermost dim contiguous on both sides, a multiple of 8, 16-byte aligned:
// one 16-byte word per thread
__global__ void __launch_bounds__(256) copy_nd_vec8(CopyArgs a) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t words = a.total / 8;
  for (uint64_t w = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += (uint64_t)gridDim.x * blockDim.x) {
    int64_t so, dof;
    cp_offsets(a, w * 8, so, dof);
    *reinterpret_cast<int4*>(a.dst + dof) = __ldg(reinterpret_cast<const int4*>(a.src + so));
  }
}

// 32 x 32 tiles over the source's unit-stride dim (is) and the destination's
// (id): reads along is, writes along id.  Block (tile_s, tile_d, outer index).
__global__ void __launch_bounds__(256) copy_nd_tiled(CopyArgs a) {
  corm_pdl_wait();
  corm_pdl_trigger();
  __shared__ int16_t tile[32][33];
  const uint32_t Ns = a.dims[a.is], Nd = a.dims[a.id];
  const uint32_t tiles_s = (Ns + 31) / 32, tiles_d = (Nd + 31) / 32;
  const uint64_t per_outer = (uint64_t)tiles_s * tiles_d;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads
  for (uint64_t blk = blockIdx.x; blk < a.outer * per_outer; blk += gridDim.x) {
    const uint64_t o = blk / per_outer;
    const uint32_t t = (uint32_t)(blk - o * per_outer);
    const uint32_t s0 = (t % tiles_s) * 32, d0 = (t / tiles_s) * 32;
    // the outer index over the other dims (row-major, is and id skipped)
    int64_t so = 0, dof = 0;
    uint64_t rem = o;
    for (int d = a.nd - 1; d >= 0; d--) {
      if (d == a.is || d == a.id) continue;
      const uint64_t q = rem / a.dims[d];
      const uint32_t x = (uint32_t)(rem - q * a.dims[d]);
      so += (int64_t)x * a.ss[d];
      dof += (int64_t)x * a.ds[d];
      rem = q;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {  // r along id, tx along is
      const uint32_t xs = s0 + tx, xd = d0 + r;
      if (xs < Ns && xd < Nd) tile[r][tx] = a.src[so + (int64_t)xs + (int64_t)xd * a.ss[a.id]];
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {  // r along is, tx along id
      const uint32_t xs = s0 + r, xd = d0 + tx;
      if (xs < Ns && xd < Nd) a.dst[dof + (int64_t)xd + (int64_t)xs * a.ds[a.is]] = tile[tx][r];
    }
  }
}

}  // namespace

extern "C" int corm_copy_nd(const corm_copy_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_copy_nd: null descriptor");
  if (d->ndim == 0 || d->ndim > (uint32_t)kMaxDims) return corm::fail(CORM_EINVAL, "corm_copy_nd: ndim %u", d->ndim);
  if (int rc = corm::check_device()) return rc;
  CopyArgs a{};
  a.src = d->src;
  a.dst = d->dst;
  a.total = 1;
  for (uint32_t i = 0; i < d->ndim; i++) {
    if (d->dims[i] == 0) return CORM_OK;
    a.total *= d->dims[i];
    if (d->dims[i] == 1) continue;
    a.dims[a.nd] = d->dims[i];
    a.ss[a.nd] = d->src_strides[i];
    a.ds[a.nd] = d->dst_strides[i];
    a.nd++;
  }
  if (!a.src || !a.dst) return corm::fail(CORM_EINVAL, "corm_copy_nd: null buffer");
  if (a.nd == 0) {  // one element
    a.nd = 1;
    a.dims[0] = 1;
    a.ss[0] = a.ds[0] = 1;
  }
  cudaStream_t st = (cudaStream_t)stream;
  const int last = a.nd - 1;
  a.is = a.id = -1;
  for (int i = 0; i < a.nd; i++) {
    if (a.ss[i] == 1 && a.is < 0) a.is = i;
    if (a.ds[i] == 1 && a.id < 0) a.id = i;
  }
  bool vec = a.ss[last] == 1 && a.ds[last] == 1 && a.dims[last] % 8 == 0 && !(((uintptr_t)a.src | (uintptr_t)a.dst) & 15u);
  for (int i = 0; i < last && vec; i++) vec = a.ss[i] % 8 == 0 && a.ds[i] % 8 == 0;
  if (vec) {
    {
      corm::ProfScope prof_("copy_nd_vec8", st);
      corm_launch_pdl(copy_nd_vec8, dim3(corm_blocks(a.total / 8, 256, 148u * 16u)), dim3(256), 0, st, a);
    }
    return corm::cuda_status("copy_nd");
  }
  if (a.is >= 0 && a.id >= 0 && a.is != a.id && a.dims[a.is] >= 8 && a.dims[a.id] >= 8) {
    a.outer = a.total / ((uint64_t)a.dims[a.is] * a.dims[a.id]);
    const uint64_t blocks = a.outer * ((a.dims[a.is] + 31) / 32) * ((a.dims[a.id] + 31) / 32);
    {
      corm::ProfScope prof_("copy_nd_tiled", st);
      corm_launch_pdl(copy_nd_tiled, dim3((unsigned)(blocks < 148u * 16u ? blocks : 148u * 16u)), dim3(256), 0, st, a);
    }
    return corm::cuda_status("copy_nd");
  }
  {
    corm::ProfScope prof_("copy_nd_elem", st);
    corm_launch_pdl(copy_nd_elem, dim3(corm_blocks(a.total, 256, 148u * 16u)), dim3(256), 0, st, a);
  }
  return corm::cuda_status("copy_nd");
}
