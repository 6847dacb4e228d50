// Host operations of the reference's LLM entries, on the device.
//
// corm_llm_attn_softmax — LlmAttnSoftmax without the softmax unit (the p12
// softmax a decode step runs on the host): phoenix367/cormorant
// inference-scheduler/src/llm_nodes.py:1532-1557 (reference) and its C twin
// llm_attn_softmax (llm_nodes.py:2978-3048).  For the query rows t < n of
// head h', keys j <= pos + t (and j > pos + t - W with a window): m = the
// max raw score, e_j = T_h[m - raw_j] (the float64 exp table of the head's
// score exponent, built on the host with libm), the sum left to right in
// float64, P_j = RNE(fl(e_j / sum) 2^f_p) saturated; every other entry 0.  A
// warp per query column: the max by shuffles, the e values staged in shared
// memory and summed in order by one lane, the P row by all lanes.
#include "corm_common.cuh"

namespace {

constexpr int kSmxWarps = 8;
constexpr int kSmxChunk = 256;  // e values staged per warp and step

__global__ void __launch_bounds__(32 * kSmxWarps) llm_smx_kernel(corm_llm_smx_desc d, uint32_t n) {
  corm_pdl_wait();
  corm_pdl_trigger();
  __shared__ double s_e[kSmxWarps][kSmxChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t GT = d.G * d.T;
  const uint64_t cols = (uint64_t)d.batch * GT;
  const uint64_t c = (uint64_t)blockIdx.x * kSmxWarps + warp;
  if (c >= cols) return;
  const uint32_t w = (uint32_t)(c % GT), hh = w / d.T, t = w % d.T;
  int16_t* out = d.p + c * d.p_stride;
  if (t >= n) {
    for (uint32_t j = lane; j < d.C; j += 32) out[j] = 0;
    return;
  }
  const uint32_t nk = d.pos + t + 1u;
  const uint32_t j0 = (d.window && nk > d.window) ? nk - d.window : 0u;
  const int16_t* col = d.s + c;  // column c of [C][s_stride]
  int32_t m = INT32_MIN;
  for (uint32_t j = j0 + lane; j < nk; j += 32) m = max(m, (int32_t)col[(uint64_t)j * d.s_stride]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  const double* tab = d.tab + (uint64_t)hh * 65536u;
  double sum = 0.0;
  for (uint32_t base = j0; base < nk; base += kSmxChunk) {
    const uint32_t cnt = min((uint32_t)kSmxChunk, nk - base);
    for (uint32_t i = lane; i < cnt; i += 32)
      s_e[warp][i] = tab[m - (int32_t)col[(uint64_t)(base + i) * d.s_stride]];
    __syncwarp();
    if (lane == 0)
      for (uint32_t i = 0; i < cnt; i++) sum += s_e[warp][i];  // in key order
    __syncwarp();
  }
  sum = __shfl_sync(0xffffffffu, sum, 0);
  const double ip = d.ip[hh];
  for (uint32_t j = lane; j < d.C; j += 32) {
    int16_t v = 0;
    if (j >= j0 && j < nk) {
      const double e = tab[m - (int32_t)col[(uint64_t)j * d.s_stride]];
      const double q = rint((e / sum) * ip);  // fl(e / sum), an exact power-of-two scale, RNE
      v = (int16_t)(q > 32767.0 ? 32767.0 : q);
    }
    out[j] = v;
  }
}

}  // namespace

extern "C" int corm_llm_attn_softmax(const corm_llm_smx_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_attn_softmax: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (!d->s || !d->p || !d->tab || !d->ip) return corm::fail(CORM_EINVAL, "corm_llm_attn_softmax: null buffer");
  if (d->T == 0 || d->G == 0 || d->C == 0 || d->batch == 0) return CORM_OK;
  if (d->Q == 0 || d->C % d->Q) return corm::fail(CORM_EINVAL, "corm_llm_attn_softmax: C %u %% Q %u", d->C, d->Q);
  if (d->s_stride < (uint64_t)d->batch * d->G * d->T || d->p_stride < d->C)
    return corm::fail(CORM_EINVAL, "corm_llm_attn_softmax: row strides below the row lengths");
  // n clamped as LlmAttention (llm_nodes.py:960-967)
  uint32_t n = d->n < d->T ? d->n : d->T;
  if (d->pos >= d->C) n = 0;
  else if (n > d->C - d->pos) n = d->C - d->pos;
  const uint64_t cols = (uint64_t)d->batch * d->G * d->T;
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("llm_smx_kernel", st);
    corm_launch_pdl(llm_smx_kernel, dim3((unsigned)((cols + kSmxWarps - 1) / kSmxWarps)), dim3(32 * kSmxWarps), 0, st, *d, n);
  }
  return corm::cuda_status("llm_attn_softmax");
}

// ---------------------------------------------------------------- greedy step
// corm_greedy_embed — the host side of a greedy decode step between two
// entries: the next token id = the first index of the largest logit of each
// sequence (LlmDequant then the caller's argmax; logits at one exponent, so
// the raw order is the value order), and its embedding row (LlmEmbed,
// llm_nodes.py:466-560: the table row as the int32 residual) for the next
// step's input.  A CTA per sequence: a strided max / first-index reduction,
// then the row copy.
namespace {

__global__ void __launch_bounds__(1024) greedy_embed_kernel(corm_greedy_desc d) {
  corm_pdl_wait();
  corm_pdl_trigger();
  __shared__ int32_t s_v[32];
  __shared__ uint32_t s_i[32];
  const uint32_t b = blockIdx.x;
  const int16_t* lg = d.logits + (uint64_t)b * d.ld;
  int32_t best = INT32_MIN;
  uint32_t bi = 0xFFFFFFFFu;
  // 8 logits per 16-byte load where the row is aligned, the rest one by one;
  // indices ascend per thread, so keeping only a strictly larger value keeps
  // the first index of a tie
  const uint32_t nv = ((uintptr_t)lg & 15u) ? 0u : d.vocab / 8u;
#pragma unroll 4
  for (uint32_t w = threadIdx.x; w < nv; w += blockDim.x) {
    const int4 x = __ldg((const int4*)lg + w);
    const int16_t* x8 = (const int16_t*)&x;
#pragma unroll
    for (int e = 0; e < 8; e++)
      if ((int32_t)x8[e] > best) {
        best = x8[e];
        bi = 8u * w + e;
      }
  }
  for (uint32_t j = 8u * nv + threadIdx.x; j < d.vocab; j += blockDim.x) {
    const int32_t v = lg[j];
    if (v > best || (v == best && j < bi)) {
      best = v;
      bi = j;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const int32_t v2 = __shfl_xor_sync(0xffffffffu, best, o);
    const uint32_t i2 = __shfl_xor_sync(0xffffffffu, bi, o);
    if (v2 > best || (v2 == best && i2 < bi)) {
      best = v2;
      bi = i2;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    s_v[threadIdx.x >> 5] = best;
    s_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  best = s_v[0];
  bi = s_i[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); w++)
    if (s_v[w] > best || (s_v[w] == best && s_i[w] < bi)) {
      best = s_v[w];
      bi = s_i[w];
    }
  if (threadIdx.x == 0 && d.ids) d.ids[b] = (int32_t)bi;
  const int32_t* row = d.table + (uint64_t)bi * d.dim;
  int32_t* out = d.out + (uint64_t)b * d.dim;
  for (uint32_t j = threadIdx.x; j < d.dim; j += blockDim.x) out[j] = row[j];
}

}  // namespace

extern "C" int corm_greedy_embed(const corm_greedy_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_greedy_embed: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (d->batch == 0) return CORM_OK;
  if (!d->logits || !d->table || !d->out || d->vocab == 0 || d->ld < d->vocab)
    return corm::fail(CORM_EINVAL, "corm_greedy_embed: null buffer or row stride below the vocabulary");
  cudaStream_t st = (cudaStream_t)stream;
  {
    corm::ProfScope prof_("greedy_embed_kernel", st);
    corm_launch_pdl(greedy_embed_kernel, dim3(d->batch), dim3(1024), 0, st, *d);
  }
  return corm::cuda_status("greedy_embed");
}

// ---------------------------------------------------------------- decode attention
// corm_llm_decode_attn — one decode step's attention of every KV group and
// sequence in one launch (a CTA per (sequence, group)): the q.K^T of the
// group's G query heads (LlmAttnConvNode "qk": the exact int16 sum, int32
// wrap, floor / 2^8, sat16), the host's p12 softmax of each head (as
// llm_smx_kernel), the P.V (LlmAttnConvNode "pv", the same rule), written
// straight into the merged rows (LlmAttnMergeNode).  Only the keys the
// softmax reads are scored (P is 0 elsewhere, so the P.V sums are the same).
namespace {

__device__ __forceinline__ int16_t kernel_out16(long long acc) {
  const int32_t w = (int32_t)(uint32_t)(unsigned long long)acc;  // the int32 accumulator wraps
  const int32_t y = w >> 8;                                       // floor / 2^8
  return (int16_t)(y > 32767 ? 32767 : (y < -32768 ? -32768 : y));
}

// HDT: the head dimension at compile time (64), or 0 (d.HD at run time).
// With HDT a key's K row is one straight run of 16-byte loads (all in flight
// at once).  Every form loads its first V rows of the P.V before the softmax,
// so that their latency hides under the softmax's serial float64 sum.  At
// most 3 heads a group: three CTAs an SM (80 registers), so that a decode
// step's (sequence, group) CTAs (64 x 5 for the 360M shape) run in one wave.
// (Holding a thread's first two K rows in registers across the AttnPrep
// needs 110 registers, two CTAs an SM, two waves: 8 decode layers 1.00
// against 0.93 ms.)
template <int G, int HDT>
__global__ void __launch_bounds__(256, G <= 3 ? 3 : 2) decode_attn_kernel(corm_llm_decode_attn_desc d, uint32_t n, uint32_t nk,
                                                          uint32_t j0) {
  corm_pdl_wait();
  corm_pdl_trigger();
  extern __shared__ __align__(16) uint8_t da_sm[];
  const uint32_t HD = HDT ? (uint32_t)HDT : d.HD, C = d.C;
  const uint32_t b = blockIdx.x % d.B, g = blockIdx.x / d.B;
  const uint32_t span = nk - j0;                       // keys the softmax reads
  int32_t* q = (int32_t*)da_sm;                        // [HD][G] (16-byte aligned: HD G 4 % 32 == 0)
  double* e = (double*)(q + HD * G);                   // [G][span]
  double* sums = e + (size_t)G * span;                 // [G]
  int16_t* S = (int16_t*)(sums + G);                   // [G][span] scores, then P
  __shared__ int32_t s_max[8][8];
  __shared__ long long s_acc[1024];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int16_t* Kw = d.kc + ((uint64_t)g * d.B + b) * C * HD;
  int16_t* Vw = d.vc + ((uint64_t)g * d.B + b) * C * HD;
  const uint32_t ut = (uint32_t)tid;
  constexpr int NW = HDT ? HDT / 8 : 1;  // 16-byte words of a K row
  int4 kA[NW];  // HDT: the K row of the key being scored
  auto load_k = [&](int4 (&w)[NW], uint32_t jj) {
    const int4* kr = (const int4*)(Kw + (uint64_t)(j0 + jj) * HD);
#pragma unroll
    for (int i = 0; i < NW; i++) w[i] = kr[i];
  };
  if (d.prep & 1u) {
    // the step's AttnPrep: RoPE of this group's k row and of its G q heads (the
    // cos / sin row of pos), v re-rounded, the new cache rows written
    const uint32_t half = HD / 2;
    const int32_t* cs_row = d.rope + (uint64_t)d.pos * 2u * HD;
    const int16_t* k0 = d.k0 + (uint64_t)b * d.ldk + g * HD;
    const int16_t* v0 = d.v0 + (uint64_t)b * d.ldv + g * HD;
    for (uint32_t i = tid; i < (G + 2) * HD; i += blockDim.x) {
      const uint32_t dd = i % HD, part = i / HD;  // parts 0 .. G-1: q heads, G: k, G + 1: v
      if (part <= (uint32_t)G && n == 0) {
        if (part < (uint32_t)G) q[dd * G + part] = 0;  // no valid row: a zero image
        continue;
      }
      if (part == (uint32_t)G + 1) {
        if (n == 0) continue;
        const int16_t x = v0[dd];
        int16_t y = x;
        if (!(d.prep & 16u)) {
          const uint8_t* e = (const uint8_t*)d.pv + 16u * ((d.prep & 8u) ? 0u : g * HD + dd);
          int32_t bq;
          memcpy(&bq, e + 4, 4);
          bq = (int32_t)((uint32_t)bq << 10) >> 10;
          const __int128 sum = ((__int128)x << (e[8] & 63u)) + (__int128)bq;
          y = (int16_t)corm_sat16_128(corm_rne_shr128(sum, (int)(e[10] & 63u)));
        }
        Vw[(uint64_t)d.pos * HD + dd] = y;
        continue;
      }
      const bool is_k = part == (uint32_t)G;
      const int16_t* src = is_k ? k0 : d.q0 + (uint64_t)b * d.ldq + (g * G + part) * HD;
      const uint32_t col = is_k ? g * HD + dd : (g * G + part) * HD + dd;
      const uint8_t* e = (const uint8_t*)(is_k ? d.pk : d.pq) +
                         16u * ((d.prep & (is_k ? 4u : 2u)) ? 0u : col);
      const int64_t x = src[dd];
      const int64_t rot = dd < half ? -(int64_t)src[dd + half] : (int64_t)src[dd - half];
      const __int128 sum = ((__int128)(x * cs_row[dd]) << (e[8] & 63u)) +
                           ((__int128)(rot * cs_row[HD + dd]) << (e[9] & 63u));
      const int16_t y = (int16_t)corm_sat16_128(corm_rne_shr128(sum, (int)(e[10] & 63u)));
      if (is_k)
        Kw[(uint64_t)d.pos * HD + dd] = y;
      else
        q[dd * G + part] = y;
    }
  } else {
    const int16_t* qx = d.qx + ((uint64_t)g * d.B + b) * HD * G;
    for (uint32_t i = tid; i < HD * G; i += blockDim.x) q[i] = qx[i];
  }
  __syncthreads();  // the new cache rows and the q image visible to the block
  const int16_t* K = Kw;
  const int16_t* V = Vw;
  int16_t* out = d.o + (uint64_t)b * d.o_stride + (uint64_t)g * G * HD;
  if (n == 0) {  // no valid row: P = 0, so every P.V sum is 0
    for (uint32_t i = tid; i < G * HD; i += blockDim.x) out[i] = 0;
    return;
  }
  // scores of the keys j0 .. nk - 1: a thread per key, the K row in 16-byte
  // words, each head's running maximum kept on the way
  int32_t mh[G];
#pragma unroll
  for (int h = 0; h < G; h++) mh[h] = INT32_MIN;
  auto put_scores = [&](const uint32_t* acc, uint32_t jj) {
#pragma unroll
    for (int h = 0; h < G; h++) {
      const int16_t sc = kernel_out16((long long)(int32_t)acc[h]);
      S[h * span + jj] = sc;
      mh[h] = max(mh[h], (int32_t)sc);
    }
  };
  if (HDT) {
    for (uint32_t jj = ut; jj < span; jj += blockDim.x) {
      load_k(kA, jj);
      // the sums modulo 2^32: the rule wraps the accumulator to int32 first
      uint32_t acc[G];
#pragma unroll
      for (int h = 0; h < G; h++) acc[h] = 0;
#pragma unroll
      for (int i = 0; i < NW; i++) {
        const int16_t* kv = (const int16_t*)&kA[i];
        int4 q4[2 * G];  // the q image of the word's 8 dimensions (8 G values)
#pragma unroll
        for (int t = 0; t < 2 * G; t++) q4[t] = ((const int4*)(q + 8 * i * G))[t];
        const int32_t* qv = (const int32_t*)q4;
#pragma unroll
        for (int e8 = 0; e8 < 8; e8++)
#pragma unroll
          for (int h = 0; h < G; h++) acc[h] += (uint32_t)(kv[e8] * qv[e8 * G + h]);
      }
      put_scores(acc, jj);
    }
  } else {
#pragma unroll 2
    for (uint32_t jj = tid; jj < span; jj += blockDim.x) {
      const int16_t* kr = K + (uint64_t)(j0 + jj) * HD;
      uint32_t acc[G];
#pragma unroll
      for (int h = 0; h < G; h++) acc[h] = 0;
      for (uint32_t d0 = 0; d0 < HD; d0 += 8) {
        const int4 w = *(const int4*)(kr + d0);
        const int16_t* kv = (const int16_t*)&w;
#pragma unroll
        for (int e8 = 0; e8 < 8; e8++)
#pragma unroll
          for (int h = 0; h < G; h++) acc[h] += (uint32_t)(kv[e8] * q[(d0 + e8) * G + h]);
      }
      put_scores(acc, jj);
    }
  }
#pragma unroll
  for (int h = 0; h < G; h++) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mh[h] = max(mh[h], __shfl_xor_sync(0xffffffffu, mh[h], o));
    if (lane == 0) s_max[h][warp] = mh[h];
  }
  __syncthreads();
  // P.V layout (below): a thread per 8 columns (one 16-byte V load per key)
  // and key group (256 / (HD / 8) groups, each taking every groups-th key).
  // The first VU keys of this thread's group are loaded now, in flight across
  // the softmax (plain loads: this launch wrote the row at pos, the prep above)
  constexpr int VU = 8;
  const uint32_t c8n = HD / 8, groups = blockDim.x / c8n, c8 = tid % c8n, kg = tid / c8n;
  int4 vv[VU];
#pragma unroll
  for (int u = 0; u < VU; u++) {
    const uint32_t jj = kg + u * groups;
    vv[u] = (kg < groups && jj < span) ? *(const int4*)(V + (uint64_t)(j0 + jj) * HD + c8 * 8) : make_int4(0, 0, 0, 0);
  }
  // per head: the maximum over the warps' maxima (every thread), e by the
  // head's table (the lookups of a head in flight together), the sum left to
  // right (one thread per head), P
#pragma unroll
  for (int h = 0; h < G; h++) {
    int32_t m = s_max[h][0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = max(m, s_max[h][w]);
    mh[h] = m;
  }
#pragma unroll
  for (int h = 0; h < G; h++) {
    const double* tab = d.tab + (uint64_t)(g * G + h) * 65536u;
#pragma unroll 4
    for (uint32_t jj = ut; jj < span; jj += blockDim.x) e[h * span + jj] = __ldg(tab + (mh[h] - (int32_t)S[h * span + jj]));
  }
  __syncthreads();
  if (tid < G) {
    double sum = 0.0;
#pragma unroll 8
    for (uint32_t jj = 0; jj < span; jj++) sum += e[tid * span + jj];  // in key order
    sums[tid] = sum;
  }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < G; h++) {
    const double sh = sums[h], iph = d.ip[g * G + h];
    for (uint32_t jj = ut; jj < span; jj += blockDim.x) {
      const double qv = rint((e[h * span + jj] / sh) * iph);
      S[h * span + jj] = (int16_t)(qv > 32767.0 ? 32767.0 : qv);  // P replaces the scores
    }
  }
  __syncthreads();
  // P.V: sums modulo 2^32 (the rule wraps to int32), the key groups reduced
  // in shared memory per head; VU rows in flight per thread
  uint32_t acc[G][8];
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int e8 = 0; e8 < 8; e8++) acc[h][e8] = 0;
  if (kg < groups)
    for (uint32_t base = kg; base < span; base += (uint32_t)VU * groups) {
      if (base != kg) {  // (the first rows were loaded before the softmax)
#pragma unroll
        for (int u = 0; u < VU; u++) {
          const uint32_t jj = base + u * groups;
          vv[u] = jj < span ? *(const int4*)(V + (uint64_t)(j0 + jj) * HD + c8 * 8) : make_int4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < VU; u++) {
        const uint32_t jj = base + u * groups;
        if (jj < span) {
          const int16_t* v8 = (const int16_t*)&vv[u];
#pragma unroll
          for (int h = 0; h < G; h++) {
            const int32_t pw = S[h * span + jj];
#pragma unroll
            for (int e8 = 0; e8 < 8; e8++) acc[h][e8] += (uint32_t)(pw * (int32_t)v8[e8]);
          }
        }
      }
    }
  // the key groups of a warp (lanes of one column word c8: lane % c8n) by
  // shuffles, then the 8 warps' sums through shared memory: every head at
  // once when G HD <= 256 (8 KB), else head by head
#pragma unroll
  for (int h = 0; h < G; h++)
#pragma unroll
    for (int e8 = 0; e8 < 8; e8++)
      for (uint32_t o = c8n; o < 32u; o <<= 1) acc[h][e8] += __shfl_xor_sync(0xffffffffu, acc[h][e8], o);
  uint32_t* red = (uint32_t*)s_acc;  // [warp][columns of the pass], <= 2048 words
  const uint32_t nwarp = blockDim.x >> 5;
  if (G * HD <= 256u) {
    if ((uint32_t)lane < c8n)
#pragma unroll
      for (int h = 0; h < G; h++)
#pragma unroll
        for (int e8 = 0; e8 < 8; e8++) red[warp * G * HD + h * HD + c8 * 8 + e8] = acc[h][e8];
    __syncthreads();
    for (uint32_t i = ut; i < G * HD; i += blockDim.x) {
      uint32_t t = 0;
      for (uint32_t w = 0; w < nwarp; w++) t += red[w * G * HD + i];
      out[i] = kernel_out16((long long)(int32_t)t);
    }
  } else {
#pragma unroll
    for (int h = 0; h < G; h++) {
      if ((uint32_t)lane < c8n)
#pragma unroll
        for (int e8 = 0; e8 < 8; e8++) red[warp * HD + c8 * 8 + e8] = acc[h][e8];
      __syncthreads();
      if (ut < HD) {
        uint32_t t = 0;
        for (uint32_t w = 0; w < nwarp; w++) t += red[w * HD + ut];
        out[h * HD + ut] = kernel_out16((long long)(int32_t)t);
      }
      __syncthreads();
    }
  }
}

}  // namespace

extern "C" int corm_llm_decode_attn(const corm_llm_decode_attn_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_llm_decode_attn: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if ((!d->qx && !(d->prep & 1u)) || !d->kc || !d->vc || !d->tab || !d->ip || !d->o)
    return corm::fail(CORM_EINVAL, "corm_llm_decode_attn: null buffer");
  if ((d->prep & 1u) && (!d->q0 || !d->k0 || !d->v0 || !d->rope || !d->pq || !d->pk ||
                         (!(d->prep & 16u) && !d->pv) || d->HD % 16))
    return corm::fail(CORM_EINVAL, "corm_llm_decode_attn: the fused AttnPrep needs q0 / k0 / v0, rope and entries");
  if (d->B == 0 || d->KV == 0) return CORM_OK;
  if (d->G == 0 || d->G > 8 || d->HD == 0 || d->HD % 8 || 256 % d->HD || d->HD * 4 > 1024 || d->Q == 0 ||
      d->C % d->Q || d->o_stride < (uint64_t)d->KV * d->G * d->HD)
    return corm::fail(CORM_EINVAL, "corm_llm_decode_attn: G %u (<= 8), HD %u (a divisor of 256, % 8), C %% Q",
                      d->G, d->HD);
  if (((uintptr_t)d->kc | (uintptr_t)d->vc) & 15u) return corm::fail(CORM_EINVAL, "corm_llm_decode_attn: unaligned caches");
  // one query row (T = 1, n = 1) clamped as LlmAttention: none past the cache
  const uint32_t n = d->pos >= d->C ? 0u : 1u;
  const uint32_t nk = n ? d->pos + 1u : 1u;
  const uint32_t j0 = (n && d->window && nk > d->window) ? nk - d->window : 0u;
  const size_t span = nk - j0;
  const size_t smem = d->G * span * 8 + d->G * 8 + (size_t)d->HD * d->G * 4 + d->G * span * 2 + 16;
  if (smem > 200 * 1024) return corm::fail(CORM_ELIMIT, "corm_llm_decode_attn: %zu keys beyond the shared memory", span);
  cudaStream_t st = (cudaStream_t)stream;
  auto launch = [&](auto kern) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    corm_launch_pdl(kern, dim3(d->B * d->KV), dim3(256), smem, st, *d, n, nk, j0);
  };
  {
    corm::ProfScope prof_("decode_attn_kernel", st);
    if (d->HD == 64) {
      switch (d->G) {
        case 1: launch(decode_attn_kernel<1, 64>); break;
        case 2: launch(decode_attn_kernel<2, 64>); break;
        case 3: launch(decode_attn_kernel<3, 64>); break;
        case 4: launch(decode_attn_kernel<4, 64>); break;
        case 5: launch(decode_attn_kernel<5, 64>); break;
        case 6: launch(decode_attn_kernel<6, 64>); break;
        case 7: launch(decode_attn_kernel<7, 64>); break;
        default: launch(decode_attn_kernel<8, 64>); break;
      }
    } else {
      switch (d->G) {
        case 1: launch(decode_attn_kernel<1, 0>); break;
        case 2: launch(decode_attn_kernel<2, 0>); break;
        case 3: launch(decode_attn_kernel<3, 0>); break;
        case 4: launch(decode_attn_kernel<4, 0>); break;
        case 5: launch(decode_attn_kernel<5, 0>); break;
        case 6: launch(decode_attn_kernel<6, 0>); break;
        case 7: launch(decode_attn_kernel<7, 0>); break;
        default: launch(decode_attn_kernel<8, 0>); break;
      }
    }
  }
  return corm::cuda_status("llm_decode_attn");
}
