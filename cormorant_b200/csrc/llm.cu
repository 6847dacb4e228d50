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
    llm_smx_kernel<<<(unsigned)((cols + kSmxWarps - 1) / kSmxWarps), 32 * kSmxWarps, 0, st>>>(*d, n);
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

__global__ void __launch_bounds__(256) greedy_embed_kernel(corm_greedy_desc d) {
  __shared__ int32_t s_v[8];
  __shared__ uint32_t s_i[8];
  const uint32_t b = blockIdx.x;
  const int16_t* lg = d.logits + (uint64_t)b * d.ld;
  int32_t best = INT32_MIN;
  uint32_t bi = 0xFFFFFFFFu;
  for (uint32_t j = threadIdx.x; j < d.vocab; j += blockDim.x) {
    const int32_t v = lg[j];
    if (v > best) {  // j ascends per thread: the first index of a tie stays
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
    greedy_embed_kernel<<<d->batch, 256, 0, st>>>(*d);
  }
  return corm::cuda_status("greedy_embed");
}
