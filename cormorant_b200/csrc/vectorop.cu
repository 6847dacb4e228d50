// VectorOPKernel on sm_100a: elementwise ops 0..9 with broadcast replay and the
// fused act (ALU ReLU/ReLU6 or the activation unit), and the softmax unit
// (ops 10 / 11).  Register semantics: phoenix367/cormorant
// inference-scheduler/test/host_emu.py:244-293 (kernels/vectorop_rtl/model/
// include/VectorOP.h:279-333); softmax integer specification
// inference-scheduler/src/vectorop_smx.py:50-66.
//
// HBM-bound: one thread per 8-lane output word (16 bytes), 128-bit loads and
// stores where the row base allows, the unit's activation table read through
// the read-only cache.
#include "corm_common.cuh"

namespace {

struct VopArgs {
  const int16_t* a;
  const int16_t* b;
  int16_t* c;
  uint32_t size, outer, a_inc, b_inc, c_inc, nw;  // nw = 8-lane words per row
  uint32_t op, act, alpha;
  const int16_t* table;  // unit act table (index raw + 32768) or nullptr
};

__device__ __forceinline__ int32_t vop_alu(int32_t x, int32_t y, uint32_t op) {
  switch (op) {
    case 0: return x + y;
    case 1: return x - y;
    case 2: return (x * y) >> 8;  // |x y| < 2^31; >> is floor
    case 3: return y ? (x * 256) / y : 0;  // C division truncates toward zero
    case 4: return x > 0 ? x : 0;
    case 5: return x > 0 ? (x < 1536 ? x : 1536) : 0;
    default: return x;
  }
}

__device__ __forceinline__ int32_t vop_act(int32_t r, uint32_t act, uint32_t alpha, const int16_t* __restrict__ tab) {
  if (act == 1) return r < 0 ? 0 : r;
  if (act == 2) return r < 0 ? 0 : (r > 1536 ? 1536 : r);
  if (act == 3) {  // LeakyReLU: rne(r * alpha / 2^16) for r < 0 (exact in double in the reference)
    if (r >= 0) return r;
    return (int32_t)corm_rne_shr64((int64_t)r * (int64_t)(alpha & 0xFFFFu), 16);
  }
  if (act >= 4 && act <= 6) return __ldg(tab + (r + 32768));
  return r;
}

__device__ __forceinline__ int32_t sat16i(int32_t v) { return v > 32767 ? 32767 : (v < -32768 ? -32768 : v); }

// OP and ACT are template parameters: the per-lane work is straight-line code.
template <int OP, int ACT>
__global__ void __launch_bounds__(256) vop_elementwise(VopArgs p) {
  corm_pdl_wait();
  corm_pdl_trigger();
  constexpr bool BINARY = OP <= 3;
  const uint64_t words = (uint64_t)p.outer * p.nw;
  for (uint64_t w = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; w < words; w += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t o = (uint32_t)(w / p.nw), j = (uint32_t)(w % p.nw);
    const uint32_t i0 = j * 8;
    const int16_t* ar = p.a + (size_t)o * p.a_inc + i0;
    const int16_t* br = BINARY ? p.b + (size_t)o * p.b_inc + i0 : nullptr;
    int16_t* cr = p.c + (size_t)o * p.c_inc + i0;
    const uint32_t lanes = min(8u, p.size - i0);
    // rows written in order on the hardware: a tail lane of row o survives only
    // where row o + 1's data does not land (lane index < c_inc), or in the last row
    const uint32_t lim = (o + 1 == p.outer) ? p.nw * 8 : min(p.nw * 8, max(p.c_inc, p.size));
    alignas(16) int16_t xa[8], xb[8], out[8];
    if (lanes == 8 && ((uintptr_t)ar & 15) == 0) {
      *(int4*)xa = __ldg((const int4*)ar);
    } else {
#pragma unroll
      for (int l = 0; l < 8; l++) xa[l] = l < (int)lanes ? ar[l] : 0;
    }
    if (BINARY) {
      if (lanes == 8 && ((uintptr_t)br & 15) == 0) {
        *(int4*)xb = __ldg((const int4*)br);
      } else {
#pragma unroll
        for (int l = 0; l < 8; l++) xb[l] = l < (int)lanes ? br[l] : 0;
      }
    }
#pragma unroll
    for (int l = 0; l < 8; l++) {
      int32_t r = sat16i(vop_alu(xa[l], BINARY ? xb[l] : 0, OP));
      r = vop_act(r, ACT, p.alpha, p.table);
      out[l] = l < (int)lanes ? (int16_t)r : (int16_t)0;
    }
    if (i0 + 8 <= lim && ((uintptr_t)cr & 15) == 0) {
      *(int4*)cr = *(int4*)out;
    } else {
#pragma unroll
      for (int l = 0; l < 8; l++)
        if (i0 + l < lim) cr[l] = out[l];
    }
  }
}

template <int OP>
void launch_vop_act(const VopArgs& p, uint32_t jact, unsigned blocks, cudaStream_t st) {
  switch (jact) {
    case 0: corm_launch_pdl(vop_elementwise<OP, 0>, dim3(blocks), dim3(256), 0, st, p); break;
    case 1: corm_launch_pdl(vop_elementwise<OP, 1>, dim3(blocks), dim3(256), 0, st, p); break;
    case 2: corm_launch_pdl(vop_elementwise<OP, 2>, dim3(blocks), dim3(256), 0, st, p); break;
    case 3: corm_launch_pdl(vop_elementwise<OP, 3>, dim3(blocks), dim3(256), 0, st, p); break;
    case 4: corm_launch_pdl(vop_elementwise<OP, 4>, dim3(blocks), dim3(256), 0, st, p); break;
    case 5: corm_launch_pdl(vop_elementwise<OP, 5>, dim3(blocks), dim3(256), 0, st, p); break;
    default: corm_launch_pdl(vop_elementwise<OP, 6>, dim3(blocks), dim3(256), 0, st, p); break;
  }
}

void launch_vop(const VopArgs& p, uint32_t op, uint32_t jact, unsigned blocks, cudaStream_t st) {
  corm::ProfScope prof_("vop_elementwise", st);
  switch (op) {
    case 0: launch_vop_act<0>(p, jact, blocks, st); break;
    case 1: launch_vop_act<1>(p, jact, blocks, st); break;
    case 2: launch_vop_act<2>(p, jact, blocks, st); break;
    case 3: launch_vop_act<3>(p, jact, blocks, st); break;
    case 4: launch_vop_act<4>(p, jact, blocks, st); break;
    case 5: launch_vop_act<5>(p, jact, blocks, st); break;
    case 6: corm_launch_pdl(vop_elementwise<6, 3>, dim3(blocks), dim3(256), 0, st, p); break;
    case 7: corm_launch_pdl(vop_elementwise<7, 4>, dim3(blocks), dim3(256), 0, st, p); break;
    case 8: corm_launch_pdl(vop_elementwise<8, 5>, dim3(blocks), dim3(256), 0, st, p); break;
    default: corm_launch_pdl(vop_elementwise<9, 6>, dim3(blocks), dim3(256), 0, st, p); break;
  }
}

// ---------------------------------------------------------------- softmax unit
struct SmxArgs {
  const int16_t* a;
  int16_t* c;
  uint32_t size, rows, a_inc, b_inc, W;
  uint32_t cm, cs, fp, valid0, period;
  const int32_t* tab;
  uint32_t cm8, csm8;  // cm << 8 and cs - 8 (the 32-bit path, 8 <= cs <= 39)
  uint32_t dm, dm2;    // the first d = m - x whose e is 0 (> 65535: none), dm in both halves
  uint32_t tabn;       // int32 entries of the shared table ahead of the column kernel's staging
};

__device__ __forceinline__ uint32_t smx_valid(uint32_t q, const SmxArgs& p) {
  const uint32_t v = p.valid0 + (p.period ? q % p.period : 0u);
  return v < p.size ? v : p.size;
}

// e = TAB[y mod 4096] >> (y div 4096), 0 when the shift reaches 63
__device__ __forceinline__ int64_t smx_e(int32_t m, int32_t x, const SmxArgs& p) {
  const uint64_t y = ((uint64_t)(uint32_t)(m - x) * (uint64_t)p.cm) >> p.cs;
  const uint64_t sh = y >> 12;
  return sh >= 63 ? 0 : ((int64_t)__ldg(p.tab + (y & 4095u)) >> sh);
}

__device__ __forceinline__ int16_t smx_p(int64_t e, uint64_t R, const SmxArgs& p) {
  const uint64_t q = ((uint64_t)e * R + (1ull << (39u - p.fp))) >> (40u - p.fp);
  return (int16_t)(q > 32767u ? 32767u : q);
}

// reductions over groups of WIDTH consecutive lanes (WIDTH <= 32, a power of 2)
template <int WIDTH, typename T>
__device__ __forceinline__ T warp_reduce_max(T v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) {
    T u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  return v;
}
template <int WIDTH>
__device__ __forceinline__ int64_t warp_reduce_sum(int64_t v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// e and P in 32 / 64-bit integer steps: y = (d cm) >> cs with d = m - x <
// 2^16 and cm < 2^24 (one 32 x 32 -> 64 multiply); e = TAB[y mod 4096] >>
// (y div 4096) is 0 once the shift reaches 17 (TAB <= 2^16); S <= 2^30 sums in
// 32 bits; R = 2^40 / S < 2^25 (S >= TAB[0] when a lane is valid), so e R <
// 2^41 is one 32 x 32 -> 64 multiply.
__device__ __forceinline__ uint32_t smx_e32(int32_t m, int32_t x, uint32_t cm, uint32_t cs, const int32_t* tab) {
  const uint64_t y = ((uint64_t)(uint32_t)(m - x) * cm) >> cs;
  const uint32_t yc = (uint32_t)min(y, (uint64_t)(17u << 12) - 1u);  // the table read is unconditional
  const uint32_t e = (uint32_t)tab[yc & 4095u] >> (yc >> 12);
  return y >= (17ull << 12) ? 0u : e;
}

// R = floor(2^40 / S) for a row sum 1 <= S < 2^32, without a 64-bit integer
// division (a long instruction sequence that every lane of a row's group
// runs, a large share of a short row's work).  q = 2^40 / S rounded to
// nearest in double lies within half an ulp (at most 2^-13) of the exact
// quotient; rounding is monotone and every integer below 2^53 is a double, so
// floor(q) is floor(2^40 / S) or one more, and one product test fixes it
// (r S <= 2^40 + S < 2^64).
__device__ __forceinline__ uint64_t smx_r40(uint32_t S) {
  uint64_t r = (uint64_t)(1099511627776.0 / (double)S);
  if (r * (uint64_t)S > (1ull << 40)) r--;
  return r;
}

__device__ __forceinline__ int16_t smx_p32(uint32_t e, uint32_t R, uint64_t rnd, uint32_t sh) {
  const uint64_t q = ((uint64_t)e * R + rnd) >> sh;
  return (int16_t)(q > 32767u ? 32767u : q);
}

// FC selects the arithmetic of e and P: 0 the 64-bit steps above, 1 (FC)
// both in 32-bit halves as below, 2 P alone for 8 <= f_p <= 15 with the e
// table (e by the 64-bit steps in its fill): a valid row's S >= TAB[0] =
// 2^16, so R <= 2^24 and R' = R 2^(f_p - 8) < 2^32; with sh = 40 - f_p,
// P = (e R + 2^(sh-1)) >> sh = (e R' + 2^31) >> 32, the high word of e R'
// plus bit 31 of its low word.
// The same two steps in 32-bit halves when 8 <= Cs <= 39 and 40 - f_p < 32
// (FC): y = floor(d Cm / 2^Cs) = umulhi(d 2^16, Cm 2^8) >> (Cs - 8) for
// d = m - x < 2^16 and Cm < 2^24 (both factors below 2^32, the high word is
// floor(d Cm / 2^8)); P = (e R + 2^(sh-1)) >> sh by a funnel shift (e R <
// 2^41, sh >= 9: the quotient fits 32 bits).
template <int FC>
__device__ __forceinline__ uint32_t smx_e(int32_t m, int32_t x, const SmxArgs& p, const int32_t* tab) {
  if (FC != 1) return smx_e32(m, x, p.cm, p.cs, tab);
  const uint32_t y = __umulhi((uint32_t)(m - x) << 16, p.cm8) >> p.csm8;
  const uint32_t yc = min(y, (17u << 12) - 1u);
  const uint32_t e = (uint32_t)tab[yc & 4095u] >> (yc >> 12);
  return y >= (17u << 12) ? 0u : e;
}

template <int FC>
__device__ __forceinline__ int16_t smx_pq(uint32_t e, uint32_t R, uint64_t rnd, uint32_t sh) {
  if (FC == 2) return (int16_t)min(__umulhi(e, R) + ((e * R) >> 31), 32767u);  // R = R' (below)
  if (FC == 0) return smx_p32(e, R, rnd, sh);
  const uint64_t t = (uint64_t)e * R + rnd;
  const uint32_t q = __funnelshift_r((uint32_t)t, (uint32_t)(t >> 32), sh);
  return (int16_t)min(q, 32767u);
}

// e of a score d = m - x below the row maximum.  d < 2^16 and y = floor(d Cm
// / 2^Cs) grows with d, so e is 0 for every d >= dm, the first d whose y
// reaches 17 << 12 (the host computes dm).  When dm is small (Q8.8 registers:
// dm = 3017) every e a job can produce is tabulated once per CTA in shared
// memory, s_e[d] for d < dm and s_e[dm] = 0, and an element's e is one
// packed subtract, one packed clamp and one shared-memory read (ET); the
// arithmetic above is the other path.
constexpr uint32_t kSmxEMax = 8192;  // largest dm tabulated (32 KB of shared memory)

template <int FC>
__device__ __forceinline__ void smx_fill_etab(int32_t* s_e, const SmxArgs& p, int nt) {
  for (uint32_t d = threadIdx.x; d <= p.dm; d += nt)
    s_e[d] = d < p.dm ? (int32_t)smx_e<FC>((int32_t)d, 0, p, p.tab) : 0;
}

// e of the two packed int16 scores of xw (low, high) against the packed row
// maximum m2: (m - x) mod 2^16 is m - x (0 <= m - x < 2^16), clamped to dm.
template <bool ET, int FC>
__device__ __forceinline__ void smx_e2(uint32_t m2, uint32_t xw, int32_t m, const SmxArgs& p, const int32_t* s_t,
                                       uint32_t& e0, uint32_t& e1) {
  if (ET) {
    const uint32_t di = __vminu2(__vsub2(m2, xw), p.dm2);
    e0 = (uint32_t)s_t[di & 0xFFFFu];
    e1 = (uint32_t)s_t[di >> 16];
  } else {
    e0 = smx_e<FC>(m, (int32_t)(int16_t)(xw & 0xFFFFu), p, s_t);
    e1 = smx_e<FC>(m, (int32_t)(int16_t)(xw >> 16), p, s_t);
  }
}

// Row mode, GROUP threads per row (16 / 32: a part of a warp per row; 256 /
// 1024: a CTA per row), PER elements per thread held in registers as PER / 8
// runs of 8 consecutive elements (16-byte loads and stores where the row
// allows), as packed int16 pairs: the row maximum by packed maxima, e by the
// table (ET) or the arithmetic, every masked element's e forced to 0 per
// 8-element run (a run wholly inside the valid length takes no mask), so the
// P of a masked element is 0 with no further test.  The TAB (or the e table)
// is built in shared memory once per CTA; CTAs then walk row groups.
template <int GROUP, int PER, int FC, bool ET>
__global__ void __launch_bounds__(GROUP >= 256 ? GROUP : 256) smx_rows(SmxArgs p) {
  corm_pdl_wait();
  corm_pdl_trigger();
  constexpr int NT = GROUP >= 256 ? GROUP : 256;
  constexpr int ROWS_PER_CTA = NT / GROUP;
  constexpr int V = PER / 8;
  extern __shared__ int32_t s_t[];  // ET: e by d (dm + 1 entries); else the TAB (4096)
  __shared__ uint32_t s_max[32];
  __shared__ uint32_t s_sum[32];
  if (ET)
    smx_fill_etab<FC>(s_t, p, NT);
  else
    for (int i = threadIdx.x; i < 4096; i += NT) s_t[i] = __ldg(p.tab + i);
  __syncthreads();
  const int lane_in_group = threadIdx.x % GROUP;
  const int group = threadIdx.x / GROUP;
  const uint64_t rnd = 1ull << (39u - p.fp);
  const uint32_t psh = 40u - p.fp;
  const uint32_t ngroups = (p.rows + ROWS_PER_CTA - 1) / ROWS_PER_CTA;
  // the next row's whole 16-byte words are loaded while this row is worked
  // (their loads stay in flight across the iteration)
  int4 xn[V];
  auto prefetch = [&](uint32_t rgn) {
    const uint32_t rown = rgn * ROWS_PER_CTA + group;
    const int16_t* xr = p.a + (size_t)rown * p.a_inc;
    const bool ok = rgn < ngroups && rown < p.rows && ((uintptr_t)xr & 15) == 0;
#pragma unroll
    for (int q = 0; q < V; q++) {
      const uint32_t j0 = (q * GROUP + lane_in_group) * 8;
      if (ok && j0 + 8 <= p.size) xn[q] = __ldg((const int4*)(xr + j0));
    }
  };
  prefetch(blockIdx.x);
  for (uint32_t rg = blockIdx.x; rg < ngroups; rg += gridDim.x) {
    const uint32_t row = rg * ROWS_PER_CTA + group;
    const bool live = row < p.rows;
    const uint32_t v = live ? smx_valid(row, p) : 0u;
    const int16_t* x = p.a + (size_t)row * p.a_inc;
    const bool xa = ((uintptr_t)x & 15) == 0;
    int4 xc[V];
#pragma unroll
    for (int q = 0; q < V; q++) xc[q] = xn[q];
    prefetch(rg + gridDim.x);
    uint32_t xp[PER / 2];  // packed pairs; masked elements hold INT16_MIN
    uint32_t mx = 0x80008000u;
#pragma unroll
    for (int q = 0; q < V; q++) {
      const uint32_t j0 = (q * GROUP + lane_in_group) * 8;
      if (live && xa && j0 + 8 <= v) {  // (v <= size: the word was prefetched)
        const int4 w = xc[q];
        xp[4 * q] = (uint32_t)w.x;
        xp[4 * q + 1] = (uint32_t)w.y;
        xp[4 * q + 2] = (uint32_t)w.z;
        xp[4 * q + 3] = (uint32_t)w.w;
      } else {
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const uint32_t lo = (live && j0 + e < v) ? (uint32_t)(uint16_t)x[j0 + e] : 0x8000u;
          const uint32_t hi = (live && j0 + e + 1 < v) ? (uint32_t)(uint16_t)x[j0 + e + 1] : 0x8000u;
          xp[4 * q + e / 2] = lo | (hi << 16);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; e++) mx = __vmaxs2(mx, xp[4 * q + e]);
    }
    mx = __vmaxs2(mx, __funnelshift_l(mx, mx, 16));  // both halves: the thread's maximum
#pragma unroll
    for (int o = (GROUP < 32 ? GROUP : 32) / 2; o > 0; o >>= 1) mx = __vmaxs2(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (GROUP > 32) {
      if ((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = mx;
      __syncthreads();
      for (int w = 0; w < GROUP / 32; w++) mx = __vmaxs2(mx, s_max[w]);
    }
    const int32_t m = (int32_t)(int16_t)(mx & 0xFFFFu);
    uint32_t ev[PER];
    uint32_t S = 0;
#pragma unroll
    for (int q = 0; q < V; q++) {
      const uint32_t j0 = (q * GROUP + lane_in_group) * 8;
      const bool whole = live && j0 + 8 <= v;
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        uint32_t e0, e1;
        smx_e2<ET, FC>(mx, xp[4 * q + e / 2], m, p, s_t, e0, e1);
        if (!whole) {
          e0 = (live && j0 + e < v) ? e0 : 0u;
          e1 = (live && j0 + e + 1 < v) ? e1 : 0u;
        }
        ev[8 * q + e] = e0;
        ev[8 * q + e + 1] = e1;
        S += e0 + e1;
      }
    }
#pragma unroll
    for (int o = (GROUP < 32 ? GROUP : 32) / 2; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (GROUP > 32) {
      if ((threadIdx.x & 31) == 0) s_sum[threadIdx.x >> 5] = S;
      __syncthreads();
      S = 0;
      for (int w = 0; w < GROUP / 32; w++) S += s_sum[w];
      __syncthreads();  // s_max / s_sum are rewritten by the next row
    }
    if (!live) continue;
    const uint32_t R = S > 0 ? (uint32_t)smx_r40(S) << (FC == 2 ? p.fp - 8u : 0u) : 0u;
    int16_t* out = p.c + (size_t)row * p.b_inc;
    const uint32_t lim = (row + 1 == p.rows) ? p.W : min(p.W, max(p.b_inc, p.size));
    const bool oa = ((uintptr_t)out & 15) == 0;
#pragma unroll
    for (int q = 0; q < V; q++) {
      const uint32_t j0 = (q * GROUP + lane_in_group) * 8;
      uint32_t o4[4];  // e = 0 (masked or beyond the row) gives P = 0
#pragma unroll
      for (int e = 0; e < 4; e++)
        o4[e] = (uint32_t)(uint16_t)smx_pq<FC>(ev[8 * q + 2 * e], R, rnd, psh) |
                ((uint32_t)(uint16_t)smx_pq<FC>(ev[8 * q + 2 * e + 1], R, rnd, psh) << 16);
      if (oa && j0 + 8 <= lim) {
        *(int4*)(out + j0) = make_int4((int)o4[0], (int)o4[1], (int)o4[2], (int)o4[3]);
      } else {
        const int16_t* o8 = (const int16_t*)o4;
#pragma unroll
        for (int e = 0; e < 8; e++)
          if (j0 + e < lim) out[j0 + e] = o8[e];
      }
    }
    for (uint32_t j = lane_in_group + PER * GROUP; j < lim; j += GROUP) out[j] = 0;  // tail beyond registers
  }
}

// Column mode: scores keys-major s[key][query] (row stride a_inc); a CTA
// stages 16 query columns of every key in shared memory, then writes P rows
// (one per query, size keys long) at stride b_inc.
__global__ void __launch_bounds__(256) smx_cols(SmxArgs p) {
  corm_pdl_wait();
  corm_pdl_trigger();
  extern __shared__ int16_t s_x[];  // [size][16]
  __shared__ int32_t s_m[16];
  __shared__ uint64_t s_R[16];
  __shared__ int64_t s_part[16][17];
  __shared__ int32_t s_mpart[16][17];
  const uint32_t q0 = blockIdx.x * 16;
  const int t = threadIdx.x;
  for (uint32_t idx = t; idx < p.size * 16u; idx += 256) {
    const uint32_t j = idx >> 4, qq = idx & 15;
    s_x[idx] = p.a[(size_t)j * p.a_inc + q0 + qq];
  }
  __syncthreads();
  const int qq = t & 15, kg = t >> 4;
  const uint32_t v = smx_valid(q0 + qq, p);
  int32_t m = INT32_MIN;
  for (uint32_t j = kg; j < v; j += 16) m = max(m, (int32_t)s_x[j * 16 + qq]);
  s_mpart[qq][kg] = m;
  __syncthreads();
  if (t < 16) {
    int32_t mm = INT32_MIN;
    for (int g = 0; g < 16; g++) mm = max(mm, s_mpart[t][g]);
    s_m[t] = mm;
  }
  __syncthreads();
  m = s_m[qq];
  int64_t S = 0;
  for (uint32_t j = kg; j < v; j += 16) S += smx_e(m, s_x[j * 16 + qq], p);
  s_part[qq][kg] = S;
  __syncthreads();
  if (t < 16) {
    int64_t ss = 0;
    for (int g = 0; g < 16; g++) ss += s_part[t][g];
    s_R[t] = ss > 0 ? (1ull << 40) / (uint64_t)ss : 0ull;
  }
  __syncthreads();
  for (int r = 0; r < 16; r++) {
    const uint32_t q = q0 + r;
    const uint32_t vr = smx_valid(q, p);
    const int32_t mr = s_m[r];
    const uint64_t R = s_R[r];
    int16_t* out = p.c + (size_t)q * p.b_inc;
    const uint32_t lim = (q + 1 == p.rows) ? p.W : min(p.W, max(p.b_inc, p.size));
    for (uint32_t j = t; j < lim; j += 256) out[j] = j < vr ? smx_p(smx_e(mr, s_x[j * 16 + r], p), R, p) : (int16_t)0;
  }
}

// Column mode with 16-byte loads and stores (size % 8 == 0, a_inc % 8 == 0,
// 16-byte aligned a, up to 8192 keys): tiles of QT query columns (32, or 8 for
// columns beyond 1024 keys) staged transposed in shared memory — query c's
// keys at s_x[base(c) + j], base(c) = c KP + 16 (c / 8), the skew putting the
// 8-column words of a key pair in distinct banks — then 256 / QT lanes per
// query, each lane taking WPL words of 8 keys for the max, the sum and the P
// row (held in registers with their e values while STORE_E, else read again
// from shared memory and e recomputed).  Same arithmetic as smx_cols; CTAs
// walk the tiles (the e table or the TAB built in shared memory once per CTA).
__device__ __forceinline__ uint32_t smx_tbase(uint32_t c, uint32_t KP) { return c * KP + 16u * (c >> 3); }

// A packed pair of scores with the lanes at or past the valid length v set to
// INT16_MIN (j: the low lane's key), so they never raise the maximum.
__device__ __forceinline__ uint32_t smx_mask2(uint32_t w, uint32_t j, uint32_t v) {
  if (j >= v) return 0x80008000u;
  return j + 1 < v ? w : ((w & 0xFFFFu) | 0x80000000u);
}

template <int QT, int WPL, bool STORE_E, int FC, bool ET>
__global__ void __launch_bounds__(256) smx_cols_t(SmxArgs p) {
  constexpr uint32_t LPQ = 256u / QT;  // lanes per query: 8 (QT 32) or 32 (QT 8, long columns)
  constexpr uint32_t PARTS = QT / 8;   // 8-query groups of the staging
  corm_pdl_wait();
  corm_pdl_trigger();
  extern __shared__ __align__(16) uint8_t smx_sm[];
  int32_t* s_t = (int32_t*)smx_sm;  // ET: e by d; else the TAB
  int16_t* s_x = (int16_t*)(s_t + p.tabn);
  const uint32_t KP = p.size + 8u;
  if (ET)
    smx_fill_etab<FC>(s_t, p, 256);
  else
    for (int i = threadIdx.x; i < 4096; i += 256) s_t[i] = __ldg(p.tab + i);
  const uint64_t rnd = 1ull << (39u - p.fp);
  const uint32_t psh = 40u - p.fp;
  const uint32_t tiles = (p.rows + QT - 1u) / QT;
  for (uint32_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const uint32_t q0 = tile * QT;
    // the keys any query of the tile reads: valid0 + its largest q mod period
    // (a causal mask reads about half); the rest of the staging is never used
    const uint32_t qn = min(QT - 1u, p.rows - 1u - q0);
    uint32_t tmax = 0;
    if (p.period) {
      const uint32_t t0 = q0 % p.period;
      tmax = t0 + qn >= p.period ? p.period - 1u : t0 + qn;
    }
    const uint32_t vmax = min(p.size, p.valid0 + tmax);
    __syncthreads();  // the previous tile's reads (and the table) are done
    // SU pairs of key rows per thread in flight (their loads first, then the
    // transposed stores); one for short columns, whose whole staging is one
    // pass of the CTA (four measured slower there: 128 keys 0.152 to 0.167 ms)
    constexpr uint32_t SU = STORE_E ? 1u : 4u;
    const uint32_t nidx = ((vmax + 1u) / 2u) * PARTS;
    for (uint32_t base = threadIdx.x; base < nidx; base += 256u * SU) {
      int4 w0[SU], w1[SU];
#pragma unroll
      for (uint32_t u = 0; u < SU; u++) {
        const uint32_t idx = base + 256u * u, jp = idx / PARTS, part = idx % PARTS;
        if (idx < nidx && q0 + 8u * part < p.rows) {
          const int16_t* src = p.a + (size_t)(2u * jp) * p.a_inc + q0 + 8u * part;
          w0[u] = __ldg((const int4*)src);
          w1[u] = __ldg((const int4*)(src + p.a_inc));
        }
      }
#pragma unroll
      for (uint32_t u = 0; u < SU; u++) {
        const uint32_t idx = base + 256u * u, jp = idx / PARTS, part = idx % PARTS;
        if (idx >= nidx || q0 + 8u * part >= p.rows) continue;
        const int16_t* v0 = (const int16_t*)&w0[u];
        const int16_t* v1 = (const int16_t*)&w1[u];
#pragma unroll
        for (int e = 0; e < 8; e++) {
          const uint32_t c = 8u * part + e;
          *(uint32_t*)(s_x + smx_tbase(c, KP) + 2u * jp) =
              (uint32_t)(uint16_t)v0[e] | ((uint32_t)(uint16_t)v1[e] << 16);
        }
      }
    }
    __syncthreads();
    // LPQ lanes per query, WPL words of 8 keys per lane
    const uint32_t r = (uint32_t)threadIdx.x / LPQ, sl = (uint32_t)threadIdx.x % LPQ;
    const uint32_t q = q0 + r;
    const bool live = q < p.rows;
    const uint32_t v = live ? smx_valid(q, p) : 0u;
    const int16_t* xs = s_x + smx_tbase(r, KP);
    // every key word this lane reads, masked past v (INT16_MIN) so the
    // maximum needs no test per key
    auto word = [&](int k) -> uint4 {
      const uint32_t j0 = 8u * (sl + LPQ * k);
      if (j0 >= v) return make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
      uint4 w = *(const uint4*)(xs + j0);  // j0 < v <= size: staged
      if (j0 + 8u > v) {
        w.x = smx_mask2(w.x, j0, v);
        w.y = smx_mask2(w.y, j0 + 2u, v);
        w.z = smx_mask2(w.z, j0 + 4u, v);
        w.w = smx_mask2(w.w, j0 + 6u, v);
      }
      return w;
    };
    uint4 xw[STORE_E ? WPL : 1];
    uint32_t mx = 0x80008000u;
#pragma unroll(STORE_E ? WPL : 1)
    for (int k = 0; k < WPL; k++) {
      if (8u * (sl + LPQ * k) >= v) break;
      const uint4 w = word(k);
      if constexpr (STORE_E) xw[k] = w;
      mx = __vmaxs2(__vmaxs2(mx, w.x), __vmaxs2(__vmaxs2(w.y, w.z), w.w));
    }
    mx = __vmaxs2(mx, __funnelshift_l(mx, mx, 16));
#pragma unroll
    for (int o = LPQ / 2; o > 0; o >>= 1) mx = __vmaxs2(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const int32_t m = (int32_t)(int16_t)(mx & 0xFFFFu);
    // e of the 8 keys of word k (0 past v)
    auto e8 = [&](int k, const uint4& w, uint32_t* e) {
      const uint32_t j0 = 8u * (sl + LPQ * k);
      const uint32_t pr[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int t = 0; t < 4; t++) smx_e2<ET, FC>(mx, pr[t], m, p, s_t, e[2 * t], e[2 * t + 1]);
      if (j0 + 8u > v) {
#pragma unroll
        for (int t = 0; t < 8; t++) e[t] = j0 + t < v ? e[t] : 0u;
      }
    };
    uint32_t ev[STORE_E ? WPL * 8 : 1];
    uint32_t S = 0;
#pragma unroll(STORE_E ? WPL : 1)
    for (int k = 0; k < WPL; k++) {
      if (8u * (sl + LPQ * k) >= v) break;
      uint32_t e[8];
      if constexpr (STORE_E)
        e8(k, xw[k], e);
      else
        e8(k, word(k), e);
#pragma unroll
      for (int t = 0; t < 8; t++) {
        if constexpr (STORE_E) ev[k * 8 + t] = e[t];
        S += e[t];
      }
    }
#pragma unroll
    for (int o = LPQ / 2; o > 0; o >>= 1) S += __shfl_xor_sync(0xffffffffu, S, o);
    if (live) {
      const uint32_t R = S > 0 ? (uint32_t)smx_r40(S) << (FC == 2 ? p.fp - 8u : 0u) : 0u;
      int16_t* out = p.c + (size_t)q * p.b_inc;
      const uint32_t lim = (q + 1 == p.rows) ? p.W : min(p.W, max(p.b_inc, p.size));
      const bool oa = ((uintptr_t)out & 15) == 0;
#pragma unroll(STORE_E ? WPL : 1)
      for (int k = 0; k < WPL; k++) {
        const uint32_t j0 = 8u * (sl + LPQ * k);
        if (j0 >= lim) break;
        uint32_t e[8];
        if (j0 >= v) {
#pragma unroll
          for (int t = 0; t < 8; t++) e[t] = 0u;
        } else if constexpr (STORE_E) {
#pragma unroll
          for (int t = 0; t < 8; t++) e[t] = ev[k * 8 + t];
        } else {
          e8(k, word(k), e);
        }
        uint32_t o4[4];  // e = 0 gives P = 0
#pragma unroll
        for (int t = 0; t < 4; t++)
          o4[t] = (uint32_t)(uint16_t)smx_pq<FC>(e[2 * t], R, rnd, psh) |
                  ((uint32_t)(uint16_t)smx_pq<FC>(e[2 * t + 1], R, rnd, psh) << 16);
        if (oa && j0 + 8 <= lim) {
          *(int4*)(out + j0) = make_int4((int)o4[0], (int)o4[1], (int)o4[2], (int)o4[3]);
        } else {
          const int16_t* o8 = (const int16_t*)o4;
#pragma unroll
          for (int t = 0; t < 8; t++)
            if (j0 + t < lim) out[j0 + t] = o8[t];
        }
      }
    }
  }
}

// CTAs for a persistent row-mode launch: at most 8 per SM
unsigned smx_grid(uint64_t groups) { return (unsigned)(groups < 148u * 8u ? (groups ? groups : 1) : 148u * 8u); }

template <int G, int P>
void launch_rows(const SmxArgs& p, unsigned grid, unsigned threads, int fc, cudaStream_t st) {
  const bool et = p.dm <= kSmxEMax;
  const size_t smem = et ? ((size_t)p.dm + 1) * sizeof(int32_t) : 4096 * sizeof(int32_t);
  if (et && fc == 1)
    corm_launch_pdl(smx_rows<G, P, 1, true>, dim3(grid), dim3(threads), smem, st, p);
  else if (et && fc == 2)
    corm_launch_pdl(smx_rows<G, P, 2, true>, dim3(grid), dim3(threads), smem, st, p);
  else if (et)
    corm_launch_pdl(smx_rows<G, P, 0, true>, dim3(grid), dim3(threads), smem, st, p);
  else if (fc == 1)
    corm_launch_pdl(smx_rows<G, P, 1, false>, dim3(grid), dim3(threads), smem, st, p);
  else
    corm_launch_pdl(smx_rows<G, P, 0, false>, dim3(grid), dim3(threads), smem, st, p);
}

// The first d = m - x (0 <= d < 2^16) with floor(d Cm / 2^Cs) >= 17 << 12, so
// e = 0 from there on; 65536 when no such d exists.
uint32_t smx_dm(uint32_t cm, uint32_t cs) {
  if (cm == 0) return 65536u;
  const unsigned __int128 need = (unsigned __int128)(17u << 12) << cs;  // d Cm >= need
  const unsigned __int128 d = (need + cm - 1) / cm;
  return d > 65536u ? 65536u : (uint32_t)d;
}

int launch_softmax(const corm_vectorop_desc* d, cudaStream_t st, const corm::DeviceTables* tb) {
  SmxArgs p{};
  p.a = d->a;
  p.c = d->c;
  p.size = d->size;
  p.a_inc = d->a_inc;
  p.b_inc = d->b_inc;
  p.W = (d->size + 7u) / 8u * 8u;
  p.cm = d->smx_cm & 0xFFFFFFu;
  p.cs = d->smx_cfg & 63u;
  p.fp = (d->smx_cfg >> 8) & 31u;
  p.valid0 = d->smx_mask & 0xFFFFu;
  p.period = d->smx_mask >> 16;
  p.tab = tb->smx_tab;
  p.cm8 = p.cm << 8;
  p.csm8 = p.cs >= 8u ? p.cs - 8u : 0u;
  p.dm = smx_dm(p.cm, p.cs);
  p.dm2 = p.dm <= 0xFFFFu ? p.dm * 0x10001u : 0xFFFFFFFFu;
  const int fc = (p.dm <= kSmxEMax && p.fp >= 8u && p.fp <= 15u) ? 2
                 : (p.cs >= 8u && p.cs <= 39u && 40u - p.fp < 32u) ? 1 : 0;
  const bool col = d->op == 11;
  p.rows = col ? (d->outer & ~15u) : d->outer;
  if (p.rows == 0) return CORM_OK;
  if (p.rows > 1 && p.b_inc < p.size)
    return corm::fail(CORM_EINVAL, "softmax: output rows overlap (b_inc %u < size %u)", p.b_inc, p.size);
  if (col && d->size % 8 == 0 && d->size <= 8192 && d->a_inc % 8 == 0 && !((uintptr_t)d->a & 15u)) {
    // 32 queries per tile up to 1024 keys; 8 (a warp per query) for longer columns
    const uint32_t qt = d->size <= 1024 ? 32u : 8u;
    const bool et = p.dm <= kSmxEMax;
    p.tabn = et ? (p.dm + 1u + 3u) / 4u * 4u : 4096u;  // keeps the staging 16-byte aligned
    const size_t smem = (size_t)p.tabn * sizeof(int32_t) +
                        (qt * ((size_t)d->size + 8) + 16 * (qt / 8)) * sizeof(int16_t);
    const uint32_t tiles = (p.rows + qt - 1) / qt;
    const unsigned per_sm = smem <= 56u * 1024u ? 4u : (smem <= 112u * 1024u ? 2u : 1u);
    const unsigned grid = tiles < 148u * per_sm ? tiles : 148u * per_sm;
    auto launch = [&](auto k_fe, auto k_he, auto k_se, auto k_f, auto k_s) {
      auto run = [&](auto kern) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        corm_launch_pdl(kern, dim3(grid), dim3(256), smem, st, p);
      };
      if (et && fc == 1) run(k_fe);
      else if (et && fc == 2) run(k_he);
      else if (et) run(k_se);
      else if (fc == 1) run(k_f);
      else run(k_s);
    };
#define CORM_SMX_COLS(Q, W, SE) \
  launch(smx_cols_t<Q, W, SE, 1, true>, smx_cols_t<Q, W, SE, 2, true>, smx_cols_t<Q, W, SE, 0, true>, \
         smx_cols_t<Q, W, SE, 1, false>, smx_cols_t<Q, W, SE, 0, false>)
    {
      corm::ProfScope prof_("smx_cols_t", st);
      if (d->size <= 64) CORM_SMX_COLS(32, 1, true);
      else if (d->size <= 128) CORM_SMX_COLS(32, 2, true);
      else if (d->size <= 256) CORM_SMX_COLS(32, 4, true);
      else if (d->size <= 512) CORM_SMX_COLS(32, 8, false);
      else if (d->size <= 1024) CORM_SMX_COLS(32, 16, false);
      else if (d->size <= 2048) CORM_SMX_COLS(8, 8, false);
      else if (d->size <= 4096) CORM_SMX_COLS(8, 16, false);
      else CORM_SMX_COLS(8, 32, false);
    }
#undef CORM_SMX_COLS
    return corm::cuda_status("softmax_cols");
  }
  if (col) {
    const size_t smem = (size_t)d->size * 16 * sizeof(int16_t);
    if (smem > 200 * 1024) return corm::fail(CORM_ELIMIT, "softmax column mode: %u keys beyond 6400", d->size);
    cudaFuncSetAttribute(smx_cols, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    {
      corm::ProfScope prof_("smx_cols", st);
      corm_launch_pdl(smx_cols, dim3(p.rows / 16), dim3(256), smem, st, p);
    }
    return corm::cuda_status("softmax_cols");
  }
  if (d->size <= 128) {
    corm::ProfScope prof_("smx_rows<16,8>", st);
    launch_rows<16, 8>(p, smx_grid((p.rows + 15) / 16), 256, fc, st);
  } else if (d->size <= 256) {
    {
      corm::ProfScope prof_("smx_rows<32,8>", st);
      launch_rows<32, 8>(p, smx_grid((p.rows + 7) / 8), 256, fc, st);
    }
  } else if (d->size <= 384) {
    {
      corm::ProfScope prof_("smx_rows<16,24>", st);
      launch_rows<16, 24>(p, smx_grid((p.rows + 15) / 16), 256, fc, st);
    }
  } else if (d->size <= 512) {
    {
      corm::ProfScope prof_("smx_rows<32,16>", st);
      launch_rows<32, 16>(p, smx_grid((p.rows + 7) / 8), 256, fc, st);
    }
  } else if (d->size <= 768) {
    {
      corm::ProfScope prof_("smx_rows<32,24>", st);
      launch_rows<32, 24>(p, smx_grid((p.rows + 7) / 8), 256, fc, st);
    }
  } else if (d->size <= 1024) {
    {
      corm::ProfScope prof_("smx_rows<32,32>", st);
      launch_rows<32, 32>(p, smx_grid((p.rows + 7) / 8), 256, fc, st);
    }
  } else if (d->size <= 4096) {
    {
      corm::ProfScope prof_("smx_rows<256,16>", st);
      launch_rows<256, 16>(p, smx_grid(p.rows), 256, fc, st);
    }
  } else if (d->size <= 16384) {
    {
      corm::ProfScope prof_("smx_rows<1024,16>", st);
      launch_rows<1024, 16>(p, smx_grid(p.rows), 1024, fc, st);
    }
  } else {
    return corm::fail(CORM_ELIMIT, "softmax row mode: size %u beyond 16384", d->size);
  }
  return corm::cuda_status("softmax_rows");
}

}  // namespace

extern "C" int corm_vectorop(const corm_vectorop_desc* d, corm_stream_t stream) {
  if (!d) return corm::fail(CORM_EINVAL, "corm_vectorop: null descriptor");
  if (int rc = corm::check_device()) return rc;
  if (d->op > 11) return corm::fail(CORM_EINVAL, "corm_vectorop: op %u", d->op);
  if (d->act > 6) return corm::fail(CORM_EINVAL, "corm_vectorop: act %u", d->act);
  if (d->size == 0 || d->outer == 0) return CORM_OK;
  if (!d->a || !d->c || (d->op <= 3 && !d->b)) return corm::fail(CORM_EINVAL, "corm_vectorop: null operand");
  cudaStream_t st = (cudaStream_t)stream;
  const corm::DeviceTables* tb = corm::tables();
  if (!tb) return CORM_ECUDA;
  if (d->op >= 10) return launch_softmax(d, st, tb);
  VopArgs p{};
  p.a = d->a;
  p.b = d->b;
  p.c = d->c;
  p.size = d->size;
  p.outer = d->outer;
  p.a_inc = d->a_inc;
  p.b_inc = d->b_inc;
  p.c_inc = d->a_inc + d->b_inc;
  p.nw = (d->size + 7u) / 8u;
  p.op = d->op;
  p.act = d->act;
  p.alpha = d->alpha;
  const uint32_t jact = (d->op >= 6 && d->op <= 9) ? d->op - 3 : d->act;
  p.table = (jact >= 4 && jact <= 6) ? tb->act[jact] : nullptr;
  if (d->outer > 1 && p.c_inc < d->size)
    return corm::fail(CORM_EINVAL, "corm_vectorop: output rows overlap (a_inc + b_inc = %u < size %u)", p.c_inc,
                      d->size);
  const uint64_t words = (uint64_t)p.outer * p.nw;
  const unsigned blocks = corm_blocks(words, 256, 148u * 16u);
  launch_vop(p, d->op, jact, blocks, st);
  return corm::cuda_status("vectorop");
}
