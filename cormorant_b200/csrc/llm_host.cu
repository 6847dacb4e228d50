// The float host operations of the reference's LLM entries, on the device:
// phoenix367/cormorant inference-scheduler/src/llm_nodes.py — LlmEmbed
// (:466-570), LlmResAdd (:572-603), LlmRMSNorm (:618-694), LlmSiluMul /
// LlmGeluMul (:697-791), LlmAttnPrep's host form (:1012-1169), LlmDequant
// (:1722-1750).  Their reference() methods compute in float64 in a fixed
// order and write results back with dtype.quantize_exp (round half to even
// at 2^-f, saturate, NaN -> 0; dtype.py:278-285) or as float32.  Every
// product, sum, quotient and square root here is an explicit IEEE
// round-to-nearest operation (__dmul_rn, __dadd_rn, __ddiv_rn, __dsqrt_rn):
// no contraction into fused multiply-adds, so each result is the float64
// value numpy computes, bit for bit.  Sums whose order matters (the squares
// of an RMSNorm row, np.cumsum's left-to-right order) are formed by one lane
// in element order from products staged in shared memory.
#include <algorithm>

#include "corm_common.cuh"

namespace {

// 2^f as an exact double (|f| < 1023)
__device__ __forceinline__ double pow2(int f) { return __longlong_as_double((long long)(1023 + f) << 52); }

// dtype.quantize_exp: RNE(v 2^f) saturated to int16, NaN -> 0 (the scaling by a
// power of two is exact, or rounds once as numpy's product does)
__device__ __forceinline__ int16_t host_st(double v, int f) {
  if (isnan(v)) return 0;
  const double r = rint(__dmul_rn(v, pow2(f)));
  return (int16_t)(r > 32767.0 ? 32767.0 : (r < -32768.0 ? -32768.0 : r));
}

// ---------------------------------------------------------------- LlmEmbed
// out[t][j] = table[clamp(ids[t], 0, rows - 1)][j] (times the float32 scale, a
// float32 product), as float32 rows or as the int32 residual at 2^-f (RNE,
// saturated to int32: llm_nodes.py _res32)
__global__ void __launch_bounds__(256) llm_embed_kernel(corm_llm_embed_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t total = (uint64_t)d.n * d.d;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t t = (uint32_t)(i / d.d), j = (uint32_t)(i - (uint64_t)t * d.d);
    int32_t k = d.ids[t];
    k = k < 0 ? 0 : (k >= (int32_t)d.rows ? (int32_t)d.rows - 1 : k);
    float v = d.table[(uint64_t)k * d.d + j];
    if (d.scale != 1.0f) v = __fmul_rn(v, d.scale);
    if (d.res32) {
      const double r = rint(__dmul_rn((double)v, pow2(d.f)));
      ((int32_t*)d.out)[i] = (int32_t)(r > 2147483647.0 ? 2147483647.0 : (r < -2147483648.0 ? -2147483648.0 : r));
    } else {
      ((float*)d.out)[i] = v;
    }
  }
}

// ---------------------------------------------------------------- LlmDequant
__global__ void __launch_bounds__(256) llm_dequant_kernel(corm_llm_dequant_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < d.count; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(i % d.n);
    d.y[i] = __double2float_rn(__dmul_rn((double)d.x[i], pow2(-(int)d.f[c])));
  }
}

// ---------------------------------------------------------------- LlmResAdd
// y = float32((double) h + d 2^-fd[c])
__global__ void __launch_bounds__(256) llm_resadd_kernel(corm_llm_resadd_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t total = (uint64_t)d.rows * d.n;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(i % d.n);
    const double dv = __dmul_rn((double)d.d[i], pow2(-(int)d.fd[c]));
    d.y[i] = __double2float_rn(__dadd_rn((double)d.h[i], dv));
  }
}

// ---------------------------------------------------------------- LlmRMSNorm
// A warp per row of n: the squares h h formed by all lanes, summed left to
// right by lane 0 (np.cumsum's order), r = 1 / sqrt(ss / n + eps), then
// y = (h r) gamma written back at the output's exponent.  h is float32 (the
// residual) or int16 at per-channel exponents (rows of W = a whole number of
// rows of n: the heads of a head norm; channel c of a row of W).
constexpr int kNormWarps = 4;
constexpr uint32_t kNormChunk = 256;

__device__ __forceinline__ double norm_h(const corm_llm_rmsnorm_desc& d, uint64_t row, uint32_t j) {
  const uint64_t idx = row * d.n + j;
  if (d.h32) return (double)d.h32[idx];
  const uint32_t c = (uint32_t)(idx % d.W);
  return __dmul_rn((double)d.h16[idx], pow2(-(int)d.fh[c]));
}

__global__ void __launch_bounds__(32 * kNormWarps) llm_rmsnorm_kernel(corm_llm_rmsnorm_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  __shared__ double s_q[kNormWarps][kNormChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t row = (uint64_t)blockIdx.x * kNormWarps + warp;
  if (row >= d.rows) return;
  double ss = 0.0;
  for (uint32_t base = 0; base < d.n; base += kNormChunk) {
    const uint32_t cnt = min(kNormChunk, d.n - base);
    for (uint32_t i = lane; i < cnt; i += 32) {
      const double h = norm_h(d, row, base + i);
      s_q[warp][i] = __dmul_rn(h, h);
    }
    __syncwarp();
    if (lane == 0)
      for (uint32_t i = 0; i < cnt; i++) ss = __dadd_rn(ss, s_q[warp][i]);
    __syncwarp();
  }
  ss = __shfl_sync(0xffffffffu, ss, 0);
  const double r = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)d.n), d.eps)));
  for (uint32_t j = lane; j < d.n; j += 32) {
    const uint64_t idx = row * d.n + j;
    const double y = __dmul_rn(__dmul_rn(norm_h(d, row, j), r), (double)d.gamma[j]);
    d.y[idx] = host_st(y, d.fy[(uint32_t)(idx % d.W)]);
  }
}

// ---------------------------------------------------------------- LlmSiluMul / LlmGeluMul
// y = st(T_c[g_raw + 32768] u 2^-fu[c], fy[c]): T_c the float64 table (libm
// exp, built on the host) of channel c's gate exponent
__global__ void __launch_bounds__(256) llm_act_mul_kernel(corm_llm_act_mul_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t total = (uint64_t)d.rows * d.n;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(i % d.n);
    const double a = d.tab[(uint64_t)d.tab_of[c] * 65536u + (uint32_t)((int32_t)d.g[i] + 32768)];
    const double u = __dmul_rn((double)d.u[i], pow2(-(int)d.fu[c]));
    d.y[i] = host_st(__dmul_rn(a, u), d.fy[c]);
  }
}

// ---------------------------------------------------------------- LlmAttnPrep (host form)
// Per sequence b and row t < n: RoPE of q0 / k0 in float64 with the float32
// tables' row pos + t (x c + rot s, rot = [-x[half:], x[:half]]); the K row
// and the v row written into the caches' row pos + t at their exponents; the
// q image qx[g][b][d][h' T + t] = clip(RNE(RoPE(q) 2^fq[h])); image columns
// t >= n are 0.  A thread per (sequence, row, channel of q, k or v).
__device__ __forceinline__ double rope_at(const int16_t* row, const int8_t* f, uint32_t base, uint32_t d, uint32_t HD,
                                          const float* cs, const float* sn) {
  const uint32_t half = HD / 2u, dp = d < half ? d + half : d - half;
  const double x = __dmul_rn((double)row[base + d], pow2(-(int)f[base + d]));
  const double xp = __dmul_rn((double)row[base + dp], pow2(-(int)f[base + dp]));
  const double rot = d < half ? -xp : xp;
  const uint32_t k = d % half;
  return __dadd_rn(__dmul_rn(x, (double)cs[k]), __dmul_rn(rot, (double)sn[k]));
}

__global__ void __launch_bounds__(256) llm_attn_prep_host_kernel(corm_llm_prep_desc d, uint32_t n) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint32_t nq = d.H * d.HD, nk = d.KV * d.HD, per = nq + 2u * nk, G = d.H / d.KV;
  const uint64_t total = (uint64_t)d.batch * d.T * per;
  const uint32_t half = d.HD / 2u;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t ch = (uint32_t)(i % per);
    const uint64_t bt = i / per;
    const uint32_t t = (uint32_t)(bt % d.T), b = (uint32_t)(bt / d.T);
    const bool live = t < n;
    const uint32_t p = d.pos + t;
    const float* cs = d.cos + (uint64_t)(live ? p : 0u) * half;
    const float* sn = d.sin + (uint64_t)(live ? p : 0u) * half;
    if (ch < nq) {  // q: the image column of head h
      const uint32_t h = ch / d.HD, dd = ch % d.HD, g = h / G, hh = h % G;
      int16_t v = 0;
      if (live) {
        const double qr = rope_at(d.q0 + bt * d.ldq, d.fq0, h * d.HD, dd, d.HD, cs, sn);
        const double r = rint(__dmul_rn(qr, pow2(d.fq[h])));
        v = (int16_t)(r > 32767.0 ? 32767.0 : (r < -32768.0 ? -32768.0 : r));
      }
      d.qx[(((uint64_t)g * d.batch + b) * d.HD + dd) * (G * d.T) + hh * d.T + t] = v;
    } else if (live) {  // k or v into the cache row pos + t (group-major [KV][B][C][HD])
      const bool isk = ch < nq + nk;
      const uint32_t c = ch - nq - (isk ? 0u : nk), g = c / d.HD, dd = c % d.HD;
      int16_t* cache = isk ? d.kc : d.vc;
      double val;
      if (isk)
        val = rope_at(d.k0 + bt * d.ldk, d.fk0, g * d.HD, dd, d.HD, cs, sn);
      else
        val = __dmul_rn((double)d.v[bt * d.ldv + c], pow2(-(int)d.fv[c]));
      cache[(((uint64_t)g * d.batch + b) * d.C + p) * d.HD + dd] = host_st(val, isk ? d.fkc[c] : d.fvc[c]);
    }
  }
}

unsigned grid_of(uint64_t work) { return corm_blocks(work, 256, 148u * 16u); }

}  // namespace

extern "C" int corm_llm_embed(const corm_llm_embed_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_embed: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (!d->ids || !d->table || !d->out || d->rows == 0)
    return corm::fail(CORM_EINVAL, "corm_llm_embed: null buffer or empty table");
  if ((uint64_t)d->n * d->d == 0) return CORM_OK;
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_embed_kernel", st);
    corm_launch_pdl(llm_embed_kernel, dim3(grid_of((uint64_t)d->n * d->d)), dim3(256), 0, st, *d);
  }
  return corm::cuda_status("llm_embed");
}

extern "C" int corm_llm_dequant(const corm_llm_dequant_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_dequant: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (d->count == 0) return CORM_OK;
  if (!d->x || !d->y || !d->f || d->n == 0) return corm::fail(CORM_EINVAL, "corm_llm_dequant: null buffer");
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_dequant_kernel", st);
    corm_launch_pdl(llm_dequant_kernel, dim3(grid_of(d->count)), dim3(256), 0, st, *d);
  }
  return corm::cuda_status("llm_dequant");
}

extern "C" int corm_llm_resadd(const corm_llm_resadd_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_resadd: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if ((uint64_t)d->rows * d->n == 0) return CORM_OK;
  if (!d->h || !d->d || !d->y || !d->fd) return corm::fail(CORM_EINVAL, "corm_llm_resadd: null buffer");
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_resadd_kernel", st);
    corm_launch_pdl(llm_resadd_kernel, dim3(grid_of((uint64_t)d->rows * d->n)), dim3(256), 0, st, *d);
  }
  return corm::cuda_status("llm_resadd");
}

extern "C" int corm_llm_rmsnorm(const corm_llm_rmsnorm_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_rmsnorm: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (d->rows == 0) return CORM_OK;
  if ((!d->h32 == !d->h16) || (d->h16 && !d->fh) || !d->y || !d->gamma || !d->fy || d->n == 0 || d->W == 0 ||
      d->W % d->n)
    return corm::fail(CORM_EINVAL, "corm_llm_rmsnorm: one of h32 / h16 (with fh), y, gamma, fy; W a multiple of n");
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_rmsnorm_kernel", st);
    corm_launch_pdl(llm_rmsnorm_kernel, dim3((unsigned)((d->rows + kNormWarps - 1) / kNormWarps)), dim3(32 * kNormWarps),
                    0, st, *d);
  }
  return corm::cuda_status("llm_rmsnorm");
}

extern "C" int corm_llm_act_mul(const corm_llm_act_mul_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_act_mul: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if ((uint64_t)d->rows * d->n == 0) return CORM_OK;
  if (!d->g || !d->u || !d->y || !d->tab || !d->tab_of || !d->fu || !d->fy)
    return corm::fail(CORM_EINVAL, "corm_llm_act_mul: null buffer");
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_act_mul_kernel", st);
    corm_launch_pdl(llm_act_mul_kernel, dim3(grid_of((uint64_t)d->rows * d->n)), dim3(256), 0, st, *d);
  }
  return corm::cuda_status("llm_act_mul");
}

extern "C" int corm_llm_attn_prep_host(const corm_llm_prep_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_attn_prep_host: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (!d->q0 || !d->k0 || !d->v || !d->kc || !d->vc || !d->qx || !d->cos || !d->sin || !d->fq0 || !d->fk0 ||
      !d->fv || !d->fkc || !d->fvc || !d->fq)
    return corm::fail(CORM_EINVAL, "corm_llm_attn_prep_host: null buffer");
  if (d->KV == 0 || d->H % d->KV || d->HD == 0 || d->HD % 2 || d->Q == 0 || d->C % d->Q || d->batch == 0)
    return corm::fail(CORM_EINVAL, "corm_llm_attn_prep_host: heads %u / %u, head_dim %u, C %u, Q %u", d->H, d->KV,
                      d->HD, d->C, d->Q);
  // the valid rows, clamped as attn_keys clamps them (llm_nodes.py:966-975)
  uint32_t n = 0;
  if (d->pos < d->C) n = std::min(std::min(d->n, d->T), d->C - d->pos);
  const uint64_t total = (uint64_t)d->batch * d->T * (d->H * d->HD + 2u * d->KV * d->HD);
  if (total == 0) return CORM_OK;
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_attn_prep_host_kernel", st);
    corm_launch_pdl(llm_attn_prep_host_kernel, dim3(grid_of(total)), dim3(256), 0, st, *d, n);
  }
  return corm::cuda_status("llm_attn_prep_host");
}
