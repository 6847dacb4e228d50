// tcgen05 kind::i8 GEMM with the four-way int16 split (see gemm_i8x4.h).
//
// Persistent: one CTA per SM (18 warps) walks work units = (batch, 128-row
// tile, 128-column tile, K split), warp-specialised.  Plane operands (int8
// hi / lo planes split beforehand):
//   warp 0       TMA producer: per 128-byte K block, 4 tiles (A hi/lo K-major,
//                B hi/lo K-major or MN-major, 128 x 128 bytes, 128-byte swizzle,
//                no multicast) into a STAGES-deep ring that runs across units
//   warp 1       TMEM owner (512 columns) and MMA issuer: 16 tcgen05.mma
//                (128x128x32) per K block into HH / MID / LL (the K steps past
//                the job's K, zero-filled, are not issued); waits for the
//                epilogue to drain TMEM before the next unit (tmem_empty)
//   warps 2..17  epilogue, four warps per TMEM lane quarter (32 columns each):
//                tcgen05.ld of the three accumulators, int64 recombine and the
//                job's rounding rule into registers, TMEM released to the next
//                unit's MMAs, then the int16 stores — or, for a K-split unit,
//                the exact int64 sums into the split's slot of a partial-sum
//                buffer that gemm_finish_kernel adds and rounds afterwards
// int16 operands (split inside the kernel): warp 0 owns TMEM and issues the
// MMAs, warp 17 lane 0 loads the raw int16 tiles by TMA (unswizzled, 64 KB a
// stage) into the stage's own bytes, warps 1..8 split them in place into the
// swizzled planes (a named barrier between reading and writing), warps 9..16
// run the epilogue (two warps per lane quarter).
// Every mbarrier wait is bounded (sm100::mbar_wait); a timeout leaves an error
// code in the per-device error word and the CTA unwinds (in-flight TMA loads
// and MMAs waited for, TMEM freed).
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "corm_common.cuh"
#include "corm_sm100.cuh"
#include "gemm_i8x4.h"
#include "silu_q.cuh"

namespace corm {
namespace {

constexpr int BM = 128, BN = 128, BK = 128;  // BK in bytes = int8 elements
constexpr int STAGES = 3;
constexpr int TILE_BYTES = BM * BK;  // 16 KB (BM == BN)
constexpr int STAGE_BYTES = 4 * TILE_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr uint32_t TMEM_COLS = 512;
// TMEM columns: HH [0, 128), MID [128, 256), LL [256, 384); int16 operands
// with raw tiles: A buffer b (hi 32 columns, lo 32 columns) at 384 + 64 b
constexpr uint32_t A_TMEM = 384;
constexpr int NUM_SMS = 148;
// Clock cycles each bounded wait of the GEMM may take before it gives up
// (about 2 s at the B200's clocks); corm_set_wait_limit overrides it.
constexpr long long kWaitDefault = 4000000000ll;

struct EpiArgs {
  int mode;
  int16_t* out;
  uint64_t out_batch_stride;
  uint32_t ldc, rows, cols;
  uint32_t P, y_cn, y_cs, y_gs;
  uint64_t img_stride;
  const int16_t* bias;
  uint32_t flags;
  uint32_t num_kb, a_planes, b_planes, b_mn, K;
  uint32_t tiles_m, tiles_n, batch, splits, kb_per_split;
  unsigned long long* partial;
  PostOp post;
  // int16 operands for the in-kernel split (a_bs16 / b_bs16 0: one plane for every batch)
  const int16_t* a16;
  const int16_t* b16;
  uint64_t a_bs16, b_bs16;
  uint32_t lda, ldb;
  uint32_t ymode;  // the form of the rule (floor_acc)
  uint32_t cvar;   // act (0 none, 1 ReLU, 2 Clip(0,6)) * 3 + bias kind (0 none, 1 per column, 2 per row)
  uint32_t bias_rows;
  int* err;
  long long wait_limit;  // clock cycles every bounded wait may take (corm_set_wait_limit)
  // mode 2 (column groups): output columns [gc[g], gc[g + 1]) go to their own
  // row-major [batch][rows][gw[g]] buffer at element offset gbase[g] from out
  int64_t gbase[4];
  uint32_t gc[5], gw[4];
  uint32_t raw_tma;  // int16 operands: raw tiles by TMA (map_ahi: A, map_bhi: B) into the stage
  uint32_t b_tma_planes;  // with raw_tma: B from its split planes (map_bhi / map_blo), only A split here
  uint32_t a_box_rows, b_pitch;  // raw boxes: A rows (<= 128) and the B row's bytes (<= 256)
  // A in TMEM and at most 64 rows: MMAs of M = 64, whose A and accumulator
  // rows 16 q .. 16 q + 15 sit in TMEM lanes 32 q .. 32 q + 15 (lane quarter q)
  uint32_t m64;
  // gate / up pairs (GemmJob::mulact): MULACT of each 16-column gate block and
  // the up block after it, stored at column (block start) / 2
  uint32_t mulact;
  int32_t ma_sa, ma_sc;
  const uint64_t* sig;
};

// y = floor(acc / 2^8) for acc = 2^16 HH + 2^8 MID + LL + 2^8 bias, i.e.
// 2^8 HH + MID + bias + floor(LL / 2^8) (LL >= 0), saturated, then the act
// flags: in int32 when the job's K keeps every term below 2^31, else in
// int64; under CORM_F_WRAP32 acc is formed modulo 2^32 first.
__device__ __forceinline__ int32_t sat_act(int32_t y, uint32_t flags) {
  y = y > 32767 ? 32767 : (y < -32768 ? -32768 : y);
  if (flags & (CORM_F_ACT_RELU | CORM_F_ACT_RELU6)) y = y < 0 ? 0 : y;
  if ((flags & CORM_F_ACT_RELU6) && y > 1536) y = 1536;
  return y;
}

// YMODE 0: every term below 2^31 (small K), one int32 sum.  1: the sum of
// MID, floor(LL / 2^8) and the bias fits int32 (K <= 16384): 2^8 HH plus it
// in one widening multiply-add, saturated through its high word.  3: the
// general int64 form.  2: CORM_F_WRAP32, the sum modulo 2^32.
template <int YMODE>
__device__ __forceinline__ int16_t combine(uint32_t hh, uint32_t mid, uint32_t ll, int32_t bias, uint32_t flags) {
  if (YMODE == 0) return (int16_t)sat_act((int32_t)hh * 256 + (int32_t)mid + bias + ((int32_t)ll >> 8), flags);
  if (YMODE == 2) {
    const uint32_t acc = (hh << 16) + (mid << 8) + ll + ((uint32_t)bias << 8);
    return (int16_t)sat_act((int32_t)acc >> 8, flags);
  }
  if (YMODE == 1) {
    const int32_t t = (int32_t)mid + bias + ((int32_t)ll >> 8);
    const int64_t y = (int64_t)(int32_t)hh * 256 + t;
    const int32_t hi = (int32_t)(y >> 32), lo = (int32_t)y;
    const int32_t y32 = hi == (lo >> 31) ? lo : (hi < 0 ? INT32_MIN : INT32_MAX);
    return (int16_t)sat_act(y32, flags);
  }
  int64_t y = (int64_t)(int32_t)hh * 256 + (int32_t)mid + bias + ((int32_t)ll >> 8);
  y = y > 32767 ? 32767 : (y < -32768 ? -32768 : y);
  return (int16_t)sat_act((int32_t)y, flags);
}

__device__ __forceinline__ int16_t finish(int64_t acc, uint32_t flags) {
  if (flags & CORM_F_WRAP32) acc = corm_wrap32(acc);
  int64_t y = corm_sat16(acc >> 8);
  if (flags & (CORM_F_ACT_RELU | CORM_F_ACT_RELU6)) y = y < 0 ? 0 : y;
  if ((flags & CORM_F_ACT_RELU6) && y > 1536) y = 1536;
  return (int16_t)y;
}

// element (bz, r, c) of the output: its address offset (mode 0: row-major with
// batch stride; mode 1: NCHW with the y channel pattern, r = n * P + p; mode 2:
// the column's group buffer, groups of whole 32-column runs)
__device__ __forceinline__ uint64_t out_offset(const EpiArgs& ep, uint32_t bz, uint32_t r, uint32_t c) {
  if (ep.mode == 0) return (uint64_t)bz * ep.out_batch_stride + (uint64_t)r * ep.ldc + c;
  if (ep.mode == 2) {
    const int g = (c >= ep.gc[1]) + (c >= ep.gc[2]) + (c >= ep.gc[3]);
    const uint64_t w = ep.gw[g];
    return (uint64_t)ep.gbase[g] + ((uint64_t)bz * ep.rows + r) * w + (c - ep.gc[g]);
  }
  const uint32_t n = r / ep.P, p = r - n * ep.P;
  const uint64_t coff = ep.y_cn ? (uint64_t)(c % ep.y_cn) * ep.y_cs + (uint64_t)(c / ep.y_cn) * ep.y_gs
                                : (uint64_t)c * ep.y_cs;
  return (uint64_t)n * ep.img_stride + coff + p;
}

// column c's offset within an output row (mode 0: c; mode 1: the y channel pattern)
__device__ __forceinline__ uint64_t col_offset(const EpiArgs& ep, uint32_t c) {
  if (ep.mode == 0) return c;
  return ep.y_cn ? (uint64_t)(c % ep.y_cn) * ep.y_cs + (uint64_t)(c / ep.y_cn) * ep.y_gs : (uint64_t)c * ep.y_cs;
}

// The fused VectorOP job on 64 packed results: op and act are uniform per job,
// so each (op, act) pair is its own straight-line loop.
template <int N2, int OPK, int ACTK>
__device__ __forceinline__ void post64(const PostOp& q, uint32_t* v2, const uint32_t* b2) {
#pragma unroll
  for (int j = 0; j < N2; j++) {
    uint32_t packed = 0;
#pragma unroll
    for (int e = 0; e < 2; e++) {
      const int32_t y = (int16_t)(v2[j] >> (16 * e)), z = (int16_t)(b2[j] >> (16 * e));
      int32_t r = OPK == 0 ? y + z : (OPK == 1 ? y - z : (OPK == 2 ? z - y : (y * z) >> 8));
      r = r > 32767 ? 32767 : (r < -32768 ? -32768 : r);
      if (ACTK == 1) r = r < 0 ? 0 : r;
      if (ACTK == 2) r = r < 0 ? 0 : (r > 1536 ? 1536 : r);
      if (ACTK == 3 && r < 0) r = (int32_t)corm_rne_shr64((int64_t)r * (int64_t)(q.alpha & 0xFFFFu), 16);
      if (ACTK == 4) r = __ldg(q.table + (r + 32768));
      packed |= (uint32_t)(uint16_t)r << (16 * e);
    }
    v2[j] = packed;
  }
}

template <int N2, int OPK>
__device__ __forceinline__ void post_act(const PostOp& q, uint32_t* v2, const uint32_t* b2) {
  switch (q.act) {
    case 0: post64<N2, OPK, 0>(q, v2, b2); break;
    case 1: post64<N2, OPK, 1>(q, v2, b2); break;
    case 2: post64<N2, OPK, 2>(q, v2, b2); break;
    case 3: post64<N2, OPK, 3>(q, v2, b2); break;
    default: post64<N2, OPK, 4>(q, v2, b2); break;
  }
}

// N2 packed pairs of results (v2) against the operand pairs (b2)
template <int N2>
__device__ __forceinline__ void post_dispatch(const PostOp& q, uint32_t* v2, const uint32_t* b2) {
  if (q.op == 0)
    post_act<N2, 0>(q, v2, b2);
  else if (q.op == 1)
    (q.rev ? post_act<N2, 2>(q, v2, b2) : post_act<N2, 1>(q, v2, b2));
  else
    post_act<N2, 3>(q, v2, b2);
}

// the fused job's operand for NC consecutive outputs of one row (columns cb ..),
// packed in pairs; every load issued before any use
template <int NC>
__device__ __forceinline__ void post_operand(const EpiArgs& ep, uint64_t rowbase, uint32_t cb, uint32_t* b2) {
  const int16_t* bsrc = ep.post.b_mode == 0 ? ep.post.b + cb : ep.post.b + rowbase + cb;
  if (ep.post.b_mode == 2) {
    const uint32_t v = (uint16_t)__ldg(ep.post.b);
#pragma unroll
    for (int j = 0; j < NC / 2; j++) b2[j] = v | (v << 16);
  } else if ((ep.mode == 0 || ep.post.b_mode == 0) && cb + NC <= ep.cols && ((uintptr_t)bsrc & 15) == 0) {
#pragma unroll
    for (int j = 0; j < NC / 8; j++) {
      const int4 t = __ldg((const int4*)bsrc + j);
      b2[4 * j] = (uint32_t)t.x;
      b2[4 * j + 1] = (uint32_t)t.y;
      b2[4 * j + 2] = (uint32_t)t.z;
      b2[4 * j + 3] = (uint32_t)t.w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < NC; j += 2) {
      const uint32_t ca = cb + j, cc2 = cb + j + 1;
      const uint32_t lo = ca < ep.cols ? (uint16_t)post_b(ep.post, rowbase + col_offset(ep, ca), ca) : 0u;
      const uint32_t hi = cc2 < ep.cols ? (uint16_t)post_b(ep.post, rowbase + col_offset(ep, cc2), cc2) : 0u;
      b2[j / 2] = lo | (hi << 16);
    }
  }
}

// NC consecutive results of row r (columns c0 ..) to the output
template <int NC>
__device__ __forceinline__ void store_row(const EpiArgs& ep, uint32_t bz, uint32_t r, uint32_t c0, const uint32_t* v2) {
  if (ep.mode != 1) {  // row-major (mode 2: an NC-column run lies in one group)
    int16_t* dst = ep.out + out_offset(ep, bz, r, c0);
    if (c0 + NC <= ep.cols && ((uintptr_t)dst & 15) == 0) {
#pragma unroll
      for (int j = 0; j < NC / 8; j++)
        ((int4*)dst)[j] = make_int4((int)v2[4 * j], (int)v2[4 * j + 1], (int)v2[4 * j + 2], (int)v2[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < NC; j++)
        if (c0 + j < ep.cols) dst[j] = (int16_t)(v2[j / 2] >> (16 * (j & 1)));
    }
  } else {  // NCHW: the row's image and pixel once, the channel offset per column
    const uint32_t n = r / ep.P, p = r - n * ep.P;
    int16_t* base = ep.out + (uint64_t)n * ep.img_stride + p;
#pragma unroll
    for (int j = 0; j < NC; j++) {
      const uint32_t c = c0 + j;
      if (c >= ep.cols) break;
      base[col_offset(ep, c)] = (int16_t)(v2[j / 2] >> (16 * (j & 1)));
    }
  }
}

// gate / up pairs: the 16 gate values of columns cg .. cg + 15 and the 16 up
// values after them (packed pairs) -> 16 MULACT results at output column cg / 2
__device__ __forceinline__ void mulact_store(const EpiArgs& ep, uint32_t bz, uint32_t r, uint32_t cg,
                                             const uint32_t* g2, const uint32_t* u2) {
  if (cg >= ep.cols) return;
  uint32_t o2[8];
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int16_t lo = corm_mulact((int16_t)(g2[j] & 0xFFFFu), (int16_t)(u2[j] & 0xFFFFu), ep.ma_sa, ep.ma_sc, ep.sig);
    const int16_t hi = corm_mulact((int16_t)(g2[j] >> 16), (int16_t)(u2[j] >> 16), ep.ma_sa, ep.ma_sc, ep.sig);
    o2[j] = (uint32_t)(uint16_t)lo | ((uint32_t)(uint16_t)hi << 16);
  }
  int16_t* dst = ep.out + (uint64_t)bz * ep.out_batch_stride + (uint64_t)r * ep.ldc + cg / 2;
  if (((uintptr_t)dst & 15) == 0) {
    ((int4*)dst)[0] = make_int4((int)o2[0], (int)o2[1], (int)o2[2], (int)o2[3]);
    ((int4*)dst)[1] = make_int4((int)o2[4], (int)o2[5], (int)o2[6], (int)o2[7]);
  } else {
#pragma unroll
    for (int j = 0; j < 16; j++) dst[j] = (int16_t)(o2[j / 2] >> (16 * (j & 1)));
  }
}

__device__ __forceinline__ uint64_t row_base(const EpiArgs& ep, uint32_t bz, uint32_t r) {
  if (ep.mode == 0) return (uint64_t)bz * ep.out_batch_stride + (uint64_t)r * ep.ldc;
  const uint32_t n = r / ep.P;
  return (uint64_t)n * ep.img_stride + (r - n * ep.P);
}

struct Unit {
  uint32_t bz, tile_r, tile_c, kb0, kb1;
};

__device__ __forceinline__ Unit unit_of(const EpiArgs& ep, uint32_t u) {
  Unit w;
  const uint32_t s = u % ep.splits, t = u / ep.splits;
  const uint32_t per_batch = ep.tiles_m * ep.tiles_n;
  w.bz = t / per_batch;
  const uint32_t rem = t - w.bz * per_batch;
  w.tile_c = (rem / ep.tiles_m) * BN;  // row tiles fastest: consecutive CTAs share the B tile
  w.tile_r = (rem % ep.tiles_m) * BM;
  w.kb0 = s * ep.kb_per_split;
  w.kb1 = min(ep.num_kb, w.kb0 + ep.kb_per_split);
  return w;
}

// Warp roles.  Plane operands (CONV = false): warp 0 lane 0 issues the TMA
// loads, warp 1 owns TMEM and lane 0 issues the MMAs, warps 2..9 run the
// epilogue.  int16 operands (CONV = true): warp 0 owns TMEM and issues the
// MMAs, warps 1..8 split int16 tiles into the hi / lo planes in the 128-byte
// swizzled layout the MMA descriptors read, warps 9..16 run the epilogue and
// warp 17 lane 0 loads the raw int16 tiles by TMA into the stage they are
// split in (ep.raw_tma; otherwise warps 1..8 load them with plain loads).
template <bool CONV>
struct Roles {
  // epilogue warps (4 per column group, one per TMEM lane quarter) and the
  // columns each drains: 16 x 32 with plane operands, 8 x 64 beside the producers
  static constexpr int ew = CONV ? 8 : 16;
  static constexpr int wc = BN * 4 / ew;
  static constexpr int threads = CONV ? 32 + 32 * 8 + 32 * ew + 32 : 64 + 32 * ew;
  static constexpr int mma_warp = CONV ? 0 : 1;
  static constexpr int epi0 = CONV ? 9 : 2;
  static constexpr int tma_warp = CONV ? 9 + ew : 0;  // int16 operands: the raw-tile loads
  static constexpr int chunk = 16;  // TMEM columns per tcgen05.ld (register budget)
};

// 16 int16 (two 16-byte words) -> their 16 high bytes and 16 low bytes
__device__ __forceinline__ void split16_regs(const int4& w0, const int4& w1, int4& hi, int4& lo) {
  hi.x = (int)__byte_perm((uint32_t)w0.x, (uint32_t)w0.y, 0x7531);
  hi.y = (int)__byte_perm((uint32_t)w0.z, (uint32_t)w0.w, 0x7531);
  hi.z = (int)__byte_perm((uint32_t)w1.x, (uint32_t)w1.y, 0x7531);
  hi.w = (int)__byte_perm((uint32_t)w1.z, (uint32_t)w1.w, 0x7531);
  lo.x = (int)__byte_perm((uint32_t)w0.x, (uint32_t)w0.y, 0x6420);
  lo.y = (int)__byte_perm((uint32_t)w0.z, (uint32_t)w0.w, 0x6420);
  lo.z = (int)__byte_perm((uint32_t)w1.x, (uint32_t)w1.y, 0x6420);
  lo.w = (int)__byte_perm((uint32_t)w1.z, (uint32_t)w1.w, 0x6420);
}

// two int32 saturated to int16 and packed (lo in bits 0..15)
__device__ __forceinline__ uint32_t pack_sat16(int32_t lo, int32_t hi) {
  uint32_t d;
  asm("cvt.pack.sat.s16.s32 %0, %1, %2;" : "=r"(d) : "r"(hi), "r"(lo));
  return d;
}

// floor(acc / 2^8) of one element as an int32 (saturated to int32 where the
// exact value lies beyond it; the int16 saturation follows), branch-free.
// YMODE 0: one int32 sum (every term below 2^31).  1 (|MID + bias +
// floor(LL / 2^8)| < 2^29): HH clamped to [-2^22, 2^22) before the shift —
// a clamped HH puts the sum beyond 2^29 with HH's sign, so the int16 result
// is the same.  2: the sum modulo 2^32 (CORM_F_WRAP32).  3: int64.
template <int YMODE>
__device__ __forceinline__ int32_t floor_acc(uint32_t hh, uint32_t mid, uint32_t ll, int32_t bias) {
  if (YMODE == 0) return (int32_t)hh * 256 + (int32_t)mid + bias + ((int32_t)ll >> 8);
  if (YMODE == 2) return (int32_t)((hh << 16) + (mid << 8) + ll + ((uint32_t)bias << 8)) >> 8;
  if (YMODE == 1) {
    const int32_t h = min(max((int32_t)hh, -(1 << 22)), (1 << 22) - 1);
    return h * 256 + (int32_t)mid + bias + ((int32_t)ll >> 8);
  }
  const int64_t y = (int64_t)(int32_t)hh * 256 + (int64_t)(int32_t)mid + bias + ((int32_t)ll >> 8);
  return (int32_t)min(max(y, (int64_t)INT32_MIN), (int64_t)INT32_MAX);
}

// CW accumulator columns of one row -> CW / 2 packed int16 pairs: the rule
// (YMODE), the bias (BK 0 none, 1 per column — a conv's channel —, 2 the
// row's own, rowb) and the act flags (ACT 0 none, 1 ReLU, 2 Clip(0,6)) as
// straight-line code
template <int CW, int YMODE, int ACT, int BK>
__device__ __forceinline__ void combine_run(const EpiArgs& ep, const uint32_t* hh, const uint32_t* mid,
                                            const uint32_t* ll, uint32_t c0, uint32_t* out2, int32_t rowb) {
#pragma unroll
  for (int j = 0; j < CW; j += 2) {
    const int32_t b0 = BK == 2 ? rowb : ((BK == 1 && c0 + j < ep.cols) ? ep.bias[c0 + j] : 0);
    const int32_t b1 = BK == 2 ? rowb : ((BK == 1 && c0 + j + 1 < ep.cols) ? ep.bias[c0 + j + 1] : 0);
    uint32_t p = pack_sat16(floor_acc<YMODE>(hh[j], mid[j], ll[j], b0),
                            floor_acc<YMODE>(hh[j + 1], mid[j + 1], ll[j + 1], b1));
    if (ACT == 1) p = __vmaxs2(p, 0u);
    if (ACT == 2) p = __vmins2(__vmaxs2(p, 0u), 0x06000600u);
    out2[j / 2] = p;
  }
}

template <int CW, int YMODE>
__device__ __forceinline__ void combine_ab(const EpiArgs& ep, const uint32_t* hh, const uint32_t* mid,
                                           const uint32_t* ll, uint32_t c0, uint32_t* out2, int32_t rowb) {
  switch (ep.cvar) {  // act * 3 + bias kind, uniform per job
    case 0: combine_run<CW, YMODE, 0, 0>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 1: combine_run<CW, YMODE, 0, 1>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 2: combine_run<CW, YMODE, 0, 2>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 3: combine_run<CW, YMODE, 1, 0>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 4: combine_run<CW, YMODE, 1, 1>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 5: combine_run<CW, YMODE, 1, 2>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 6: combine_run<CW, YMODE, 2, 0>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 7: combine_run<CW, YMODE, 2, 1>(ep, hh, mid, ll, c0, out2, rowb); break;
    default: combine_run<CW, YMODE, 2, 2>(ep, hh, mid, ll, c0, out2, rowb); break;
  }
}

template <int CW>
__device__ __forceinline__ void combine_any(const EpiArgs& ep, const uint32_t* hh, const uint32_t* mid,
                                            const uint32_t* ll, uint32_t c0, uint32_t* out2, int32_t rowb = 0) {
  switch (ep.ymode) {
    case 0: combine_ab<CW, 0>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 1: combine_ab<CW, 1>(ep, hh, mid, ll, c0, out2, rowb); break;
    case 2: combine_ab<CW, 2>(ep, hh, mid, ll, c0, out2, rowb); break;
    default: combine_ab<CW, 3>(ep, hh, mid, ll, c0, out2, rowb); break;
  }
}

template <int CW>
__device__ __forceinline__ void tmem_ld_cw(uint32_t taddr, uint32_t* r) {
  if (CW == 32)
    sm100::tmem_ld32(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  else
    sm100::tmem_ld16(taddr, r);
}

// DIAG: the bounded waits take the host's diagnostic limit (corm_set_wait_limit)
// instead of the compile-time default.
template <bool CONV, bool DIAG>
__global__ void __launch_bounds__(Roles<CONV>::threads, 1)
    gemm_i8x4_kernel(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
                     const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
                     const EpiArgs ep) {
  using R = Roles<CONV>;
  constexpr int CW = R::chunk;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = (uint64_t*)(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tmem_full = empty + STAGES;
  uint64_t* tmem_empty = tmem_full + 1;
  uint64_t* mma_done = tmem_empty + 1;
  uint64_t* raw_full = mma_done + 1;  // int16 raw tiles landed (CONV with raw_tma)
  uint64_t* a_free = raw_full + STAGES;  // the MMAs reading TMEM A buffer 0 / 1 are done
  uint32_t* tmem_slot = (uint32_t*)(a_free + 2);
  uint32_t* abort_at = tmem_slot + 1;  // first ring step a splitting warp gave up at
  volatile int* cta_stop = (volatile int*)(abort_at + 1);  // a role of this CTA gave up (bounded waits)
  // The bounded waits: the production kernel has a compile-time limit and no
  // stop word (once one role has given up the others run out their own
  // limits; polling the word cost the MatMul sweep 7 %); the diagnostic
  // instantiation takes the host's limit and stops every role at once.
  const long long wlim = DIAG ? ep.wait_limit : kWaitDefault;
  volatile int* const wstop = DIAG ? cta_stop : nullptr;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t units = ep.batch * ep.tiles_m * ep.tiles_n * ep.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      sm100::mbar_init(&full[s], CONV ? 8 : 1);
      sm100::mbar_init(&empty[s], 1);
      if (CONV) sm100::mbar_init(&raw_full[s], 1);
    }
    if (CONV) {
      sm100::mbar_init(&a_free[0], 1);
      sm100::mbar_init(&a_free[1], 1);
    }
    if (CONV) *abort_at = 0xFFFFFFFFu;
    *cta_stop = 0;
    sm100::mbar_init(tmem_full, 1);
    sm100::mbar_init(tmem_empty, R::ew);
    sm100::mbar_init(mma_done, 1);
    sm100::fence_mbar_init();
  }
  if (warp == R::mma_warp) sm100::tmem_alloc<TMEM_COLS>(tmem_slot);
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // the prologue above overlaps the previous kernel; global memory only after
  // it.  The next kernel may launch once every CTA's epilogue reaches its last
  // unit (below): an early launch would park its CTAs beside a long GEMM.
  corm_pdl_wait();

  if (!CONV && warp == 0 && lane == 0) {
    // ---------------- TMA producer (ring counter g runs across units)
    sm100::prefetch_tmap(&map_ahi);
    sm100::prefetch_tmap(&map_alo);
    sm100::prefetch_tmap(&map_bhi);
    sm100::prefetch_tmap(&map_blo);
    uint32_t g = 0;
    bool ok = true;
    for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const Unit w = unit_of(ep, u);
      const int a_z = ep.a_planes == 1 ? 0 : (int)w.bz, b_z = ep.b_planes == 1 ? 0 : (int)w.bz;
      for (uint32_t kb = w.kb0; kb < w.kb1; kb++, g++) {
        const int s = g % STAGES;
        if (g >= (uint32_t)STAGES && !sm100::mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, ep.err, 101, wlim, wstop)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        sm100::mbar_expect_tx(&full[s], STAGE_BYTES);
        const int x = (int)(kb * BK);
        sm100::tma_load_3d(st, &map_ahi, &full[s], x, (int)w.tile_r, a_z);
        sm100::tma_load_3d(st + TILE_BYTES, &map_alo, &full[s], x, (int)w.tile_r, a_z);
        if (ep.b_mn) {  // B planes [plane][K][cols]: box = 128 columns x 128 K rows
          sm100::tma_load_3d(st + 2 * TILE_BYTES, &map_bhi, &full[s], (int)w.tile_c, x, b_z);
          sm100::tma_load_3d(st + 3 * TILE_BYTES, &map_blo, &full[s], (int)w.tile_c, x, b_z);
        } else {
          sm100::tma_load_3d(st + 2 * TILE_BYTES, &map_bhi, &full[s], x, (int)w.tile_c, b_z);
          sm100::tma_load_3d(st + 3 * TILE_BYTES, &map_blo, &full[s], x, (int)w.tile_c, b_z);
        }
      }
    }
    if (!ok) {
      // let the loads already issued land before the CTA's shared memory goes away
      for (uint32_t q = g > (uint32_t)STAGES ? g - STAGES : 0; q < g; q++)
        sm100::mbar_wait(&full[q % STAGES], (q / STAGES) & 1, nullptr, 0, 200000000ll);
    }
  } else if (CONV && warp == R::tma_warp && lane == 0 && ep.raw_tma) {
    // ---------------- raw int16 tiles by TMA: per stage the A tile (up to 128
    // rows x 128 K as two halves of 64 K, 128-byte swizzle, over the A plane
    // bytes) and the MN-major B tile (128 K rows x up to 128 columns,
    // unswizzled, over the B planes), zero-filled beyond the job
    sm100::prefetch_tmap(&map_ahi);
    sm100::prefetch_tmap(&map_bhi);
    if (ep.b_tma_planes) sm100::prefetch_tmap(&map_blo);
    uint32_t g = 0;
    bool ok = true;
    for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const Unit w = unit_of(ep, u);
      const int a_z = ep.a_bs16 ? (int)w.bz : 0, b_z = ep.b_bs16 ? (int)w.bz : 0;
      for (uint32_t kb = w.kb0; kb < w.kb1; kb++, g++) {
        const int s = g % STAGES;
        if (g >= (uint32_t)STAGES && !sm100::mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, ep.err, 106, wlim, wstop)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        const int x = (int)(kb * BK);
        if (ep.b_tma_planes) {  // B split beforehand: its hi / lo planes as the plane path loads them
          sm100::mbar_expect_tx(&raw_full[s], ep.a_box_rows * 256u + 2 * TILE_BYTES);
          const int bp_z = ep.b_planes == 1 ? 0 : (int)w.bz;
          sm100::tma_load_3d(st + 2 * TILE_BYTES, &map_bhi, &raw_full[s], (int)w.tile_c, x, bp_z);
          sm100::tma_load_3d(st + 3 * TILE_BYTES, &map_blo, &raw_full[s], (int)w.tile_c, x, bp_z);
        } else {
          sm100::mbar_expect_tx(&raw_full[s], ep.a_box_rows * 256u + BK * ep.b_pitch);
          sm100::tma_load_3d(st + 2 * TILE_BYTES, &map_bhi, &raw_full[s], (int)w.tile_c, x, b_z);
        }
        sm100::tma_load_3d(st, &map_ahi, &raw_full[s], x, (int)w.tile_r, a_z);
        sm100::tma_load_3d(st + ep.a_box_rows * 128u, &map_ahi, &raw_full[s], x + 64, (int)w.tile_r, a_z);
      }
    }
    // the loads issued land before the CTA's shared memory goes away
    for (uint32_t q = g > (uint32_t)STAGES ? g - STAGES : 0; q < g; q++)
      sm100::mbar_wait(&raw_full[q % STAGES], (q / STAGES) & 1, nullptr, 0, 200000000ll);
  } else if (CONV && warp >= 1 && warp <= 8 && ep.raw_tma) {
    // ---------------- split of the raw tiles.  A goes to tensor memory: warp w
    // owns TMEM lane quarter q = w % 4 (rows 32 q + lane) and K half hk (warps
    // 1..4: K bytes 0..63 of the block, 5..8: 64..127); each lane reads its
    // row's 8 chunks of 16 bytes from the 128-byte-swizzled raw half-tile
    // (8 consecutive rows hit 8 distinct bank groups), splits them and stores
    // 16 hi and 16 lo words with tcgen05.st into the stage's A buffer (two
    // buffers, the MMAs of stage g - 2 waited for through a_free).  B is split
    // in place: each thread reads its 8 chunks (8 consecutive int16 of a K row,
    // 16 chunks to a 256-byte raw row, 8 lanes reading 128 contiguous bytes),
    // the 256 splitting threads meet at a named barrier, then each writes the
    // chunk's 8 hi and 8 lo bytes at their swizzled plane positions (16-byte
    // unit u of row r at (u ^ (r & 7)) * 16, the chunk in its half).  A rows and
    // B columns past the job are not split: they only reach accumulator rows /
    // columns the epilogue does not store.  The decision to stop (a bounded
    // wait ran out) is read after the barrier from abort_at, so every
    // splitting thread leaves at the same ring step.
    // B chunk i of this thread: K row row0 + 16 i, chunk c of the row (the same c
    // and row & 7 for every i, so every address is a base plus a constant)
    const uint32_t pt = (uint32_t)(warp - 1) * 32u + lane, row0 = pt >> 4, c = pt & 15u;
    const uint32_t off0 = row0 * 128u + (((c >> 1) ^ (row0 & 7u)) << 4) + ((c & 1u) << 3);
    // the A row this lane puts in its TMEM lane (M = 64: lanes 16..31 of a quarter hold none)
    const uint32_t aq = (uint32_t)(warp & 3), ahk = (uint32_t)(warp - 1) >> 2;
    const uint32_t arow = ep.m64 ? aq * 16u + (lane & 15u) : aq * 32u + lane;
    const bool a_lane = !ep.m64 || lane < 16u;
    const uint32_t q_row0 = ep.m64 ? aq * 16u : aq * 32u;
    uint32_t g = 0;
    bool stop = false;
    for (uint32_t u = blockIdx.x; u < units && !stop; u += gridDim.x) {
      const Unit w = unit_of(ep, u);
      const uint32_t nrow = ep.rows - w.tile_r, ncol = ep.cols - w.tile_c;
      for (uint32_t kb = w.kb0; kb < w.kb1; kb++, g++) {
        const int s = g % STAGES;
        bool okw = sm100::mbar_wait(&raw_full[s], (g / STAGES) & 1, ep.err, 105, wlim, wstop);
        if (g >= 2) okw = sm100::mbar_wait(&a_free[g & 1], ((g >> 1) - 1) & 1, ep.err, 109, wlim, wstop) && okw;
        if (!okw) atomicMin(abort_at, g);
        sm100::tc_fence_after();  // the TMEM buffer's readers are done (a_free)
        uint8_t* st = smem + s * STAGE_BYTES;
        // (after a run-out wait the words are not used: every thread stops below)
        if (q_row0 < nrow) {  // warp-uniform: the quarter holds rows of the job
          const uint8_t* ra = st + ahk * (ep.a_box_rows * 128u) + arow * 128u;
          uint32_t hi[16], lo[16];
#pragma unroll
          for (int k = 0; k < 8; k++) {
            int4 v = make_int4(0, 0, 0, 0);
            if (a_lane && arow < nrow) v = *(const int4*)(ra + (((uint32_t)k ^ (arow & 7u)) << 4));
            hi[2 * k] = __byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x7531);
            hi[2 * k + 1] = __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x7531);
            lo[2 * k] = __byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x6420);
            lo[2 * k + 1] = __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x6420);
          }
          const uint32_t ta = tmem + ((aq * 32u) << 16) + A_TMEM + 64u * (g & 1u) + 16u * ahk;
          sm100::tmem_st16(ta, hi);
          sm100::tmem_st16(ta + 32u, lo);
        }
        if (ep.b_tma_planes) {
          // B came split: no shared-memory writes here, so no barrier between
          // the warps; a warp whose wait ran out stops as a whole (the MMA
          // warp's bounded wait on this stage then runs out too)
          if (!__all_sync(0xffffffffu, okw)) {
            stop = true;
            break;
          }
          sm100::tmem_st_wait();
          sm100::tc_fence_before();
          __syncwarp();
          if (lane == 0) sm100::mbar_arrive(&full[s]);
          continue;
        }
        int4 vb[8];
        const uint8_t* rb = st + 2 * TILE_BYTES + row0 * ep.b_pitch + c * 16u;
        const uint32_t bstep = 16u * ep.b_pitch;
        const bool b_in = c * 8u < ncol;
#pragma unroll
        for (int i = 0; i < 8; i++)
          if (b_in) vb[i] = *(const int4*)(rb + bstep * i);
        asm volatile("bar.sync 1, 256;" ::: "memory");
        if (*(volatile uint32_t*)abort_at <= g) {
          stop = true;
          break;
        }
        if (b_in) {
#pragma unroll
          for (int i = 0; i < 8; i++) {
            const uint32_t off = off0 + 2048u * i;
            const int4 v = vb[i];
            *(uint2*)(st + 2 * TILE_BYTES + off) = make_uint2(__byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x7531),
                                                              __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x7531));
            *(uint2*)(st + 3 * TILE_BYTES + off) = make_uint2(__byte_perm((uint32_t)v.x, (uint32_t)v.y, 0x6420),
                                                              __byte_perm((uint32_t)v.z, (uint32_t)v.w, 0x6420));
          }
        }
        sm100::tmem_st_wait();
        sm100::tc_fence_before();
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&full[s]);
      }
    }
  } else if (CONV && warp >= 1 && warp <= 8) {
    // ---------------- int16 producers: per stage the A tile (128 rows x 128 K)
    // and the MN-major B tile (128 K rows x 128 columns), each as 1024 units of
    // 16 consecutive int16 -> a 16-byte hi unit and a 16-byte lo unit at the
    // row's swizzled position (unit u of row r at (u ^ (r & 7)) * 16); rows,
    // K and columns beyond the job are zeros.  K and the column count are
    // multiples of 8, every base 16-byte aligned (the host checks).
    const uint32_t pt = (uint32_t)(warp - 1) * 32u + lane;
    uint32_t g = 0;
    bool ok = true;
    for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x) {
      const Unit w = unit_of(ep, u);
      const int16_t* Ab = ep.a16 + (uint64_t)w.bz * ep.a_bs16;
      const int16_t* Bb = ep.b16 + (uint64_t)w.bz * ep.b_bs16;
      for (uint32_t kb = w.kb0; kb < w.kb1; kb++, g++) {
        const int s = g % STAGES;
        if (g >= (uint32_t)STAGES && !sm100::mbar_wait(&empty[s], ((g / STAGES) - 1) & 1, ep.err, 101, wlim, wstop)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * STAGE_BYTES;
        int4 va[4][2], vb[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t id = pt + 256u * i, row = id >> 3, uu = id & 7u;
          const int4 z = make_int4(0, 0, 0, 0);
          // A row tile_r + row, K kb*128 + 16 uu ..
          const uint32_t ar = w.tile_r + row, ak = kb * BK + uu * 16u;
          const int16_t* pa = Ab + (uint64_t)ar * ep.lda + ak;
          const bool ar_ok = ar < ep.rows;
          va[i][0] = (ar_ok && ak < ep.K) ? __ldg((const int4*)pa) : z;
          va[i][1] = (ar_ok && ak + 8u < ep.K) ? __ldg((const int4*)pa + 1) : z;
          // B K row kb*128 + row, columns tile_c + 16 uu ..
          const uint32_t bk = kb * BK + row, bc = w.tile_c + uu * 16u;
          const int16_t* pb = Bb + (uint64_t)bk * ep.ldb + bc;
          const bool bk_ok = bk < ep.K;
          vb[i][0] = (bk_ok && bc < ep.cols) ? __ldg((const int4*)pb) : z;
          vb[i][1] = (bk_ok && bc + 8u < ep.cols) ? __ldg((const int4*)pb + 1) : z;
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
          const uint32_t id = pt + 256u * i, row = id >> 3, uu = id & 7u;
          const uint32_t off = row * 128u + ((uu ^ (row & 7u)) << 4);
          int4 hi, lo;
          split16_regs(va[i][0], va[i][1], hi, lo);
          *(int4*)(st + off) = hi;
          *(int4*)(st + TILE_BYTES + off) = lo;
          split16_regs(vb[i][0], vb[i][1], hi, lo);
          *(int4*)(st + 2 * TILE_BYTES + off) = hi;
          *(int4*)(st + 3 * TILE_BYTES + off) = lo;
        }
        sm100::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(&full[s]);
      }
    }
  } else if (warp == R::mma_warp && lane == 0) {
    // ---------------- MMA issuer
    const uint32_t bmaj = ep.b_mn ? (1u << 16) : 0u;
    const uint32_t mm = ep.m64 ? 64u : (uint32_t)BM;
    const uint32_t ID_SS = sm100::idesc_i8(mm, BN, 1, 1) | bmaj;
    const uint32_t ID_SU = sm100::idesc_i8(mm, BN, 1, 0) | bmaj;
    const uint32_t ID_US = sm100::idesc_i8(mm, BN, 0, 1) | bmaj;
    const uint32_t ID_UU = sm100::idesc_i8(mm, BN, 0, 0) | bmaj;
    const uint32_t acc_hh = tmem, acc_mid = tmem + BN, acc_ll = tmem + 2 * BN;
    const bool a_tm = CONV && ep.raw_tma;  // A from the TMEM buffers the splitting warps fill
    uint32_t g = 0, i = 0;
    bool ok = true;
    for (uint32_t u = blockIdx.x; u < units && ok; u += gridDim.x, i++) {
      const Unit w = unit_of(ep, u);
      if (i > 0 && !sm100::mbar_wait(tmem_empty, (i - 1) & 1, ep.err, 104, wlim, wstop)) break;
      sm100::tc_fence_after();
      for (uint32_t kb = w.kb0; kb < w.kb1; kb++, g++) {
        const int s = g % STAGES;
        if (!sm100::mbar_wait(&full[s], (g / STAGES) & 1, ep.err, 102, wlim, wstop)) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const uint32_t base = sm100::smem_u32(smem + s * STAGE_BYTES);
        const uint64_t d_ahi = sm100::sdesc_sw128(base), d_alo = sm100::sdesc_sw128(base + TILE_BYTES);
        const uint64_t d_bhi = ep.b_mn ? sm100::sdesc_sw128_mn(base + 2 * TILE_BYTES) : sm100::sdesc_sw128(base + 2 * TILE_BYTES);
        const uint64_t d_blo = ep.b_mn ? sm100::sdesc_sw128_mn(base + 3 * TILE_BYTES) : sm100::sdesc_sw128(base + 3 * TILE_BYTES);
        // K step of 32 int8: 32 bytes inside a K-major swizzled row, or 32 rows
        // (4 swizzle atoms of 1024 bytes) of an MN-major tile
        const uint64_t b_step = ep.b_mn ? (uint64_t)(4096 >> 4) : (uint64_t)(32 >> 4);
        const uint32_t krem = ep.K - kb * BK;  // > 0: K steps beyond it only add zeros
        const int nks = krem >= (uint32_t)BK ? BK / 32 : (int)((krem + 31) / 32);
        if (a_tm) {  // A hi / lo from the stage's TMEM buffer: 8 columns per K step of 32
          const uint32_t t_ahi = tmem + A_TMEM + 64u * (g & 1u), t_alo = t_ahi + 32u;
#pragma unroll
          for (int ks = 0; ks < BK / 32; ks++) {
            if (ks >= nks) break;
            const uint64_t bdv = b_step * ks;
            const uint32_t acc = (kb != w.kb0 || ks) ? 1u : 0u;
            sm100::mma_i8_ta(acc_hh, t_ahi + 8 * ks, d_bhi + bdv, ID_SS, acc);
            sm100::mma_i8_ta(acc_mid, t_ahi + 8 * ks, d_blo + bdv, ID_SU, acc);
            sm100::mma_i8_ta(acc_mid, t_alo + 8 * ks, d_bhi + bdv, ID_US, 1u);
            sm100::mma_i8_ta(acc_ll, t_alo + 8 * ks, d_blo + bdv, ID_UU, acc);
          }
        } else {
#pragma unroll
          for (int ks = 0; ks < BK / 32; ks++) {
            if (ks >= nks) break;
            const uint64_t adv = (uint64_t)((ks * 32) >> 4), bdv = b_step * ks;
            const uint32_t acc = (kb != w.kb0 || ks) ? 1u : 0u;
            sm100::mma_i8(acc_hh, d_ahi + adv, d_bhi + bdv, ID_SS, acc);
            sm100::mma_i8(acc_mid, d_ahi + adv, d_blo + bdv, ID_SU, acc);
            sm100::mma_i8(acc_mid, d_alo + adv, d_bhi + bdv, ID_US, 1u);
            sm100::mma_i8(acc_ll, d_alo + adv, d_blo + bdv, ID_UU, acc);
          }
        }
        sm100::mma_commit(&empty[s]);
        if (a_tm) sm100::mma_commit(&a_free[g & 1u]);
      }
      if (ok) sm100::mma_commit(tmem_full);
    }
    // every MMA issued has completed before TMEM is freed
    sm100::mma_commit(mma_done);
    sm100::mbar_wait(mma_done, 0, nullptr, 0, 200000000ll);
  } else if (warp >= R::epi0 && (!CONV || warp < R::epi0 + R::ew)) {
    // ---------------- epilogue: warp (epi0 + 4 h + j) reads lane quarter (warp % 4),
    // columns [64 h, 64 h + 64)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    const int h = (warp - R::epi0) >> 2;
    uint32_t i = 0;
    for (uint32_t u = blockIdx.x; u < units; u += gridDim.x, i++) {
      const Unit w = unit_of(ep, u);
      if (u + gridDim.x >= units) corm_pdl_trigger();  // this CTA's last unit
      const uint32_t r = w.tile_r + (ep.m64 ? q * 16 + (lane & 15) : q * 32 + lane);
      const bool row_ok = (!ep.m64 || lane < 16) && r < ep.rows;
      // a per-row bias (a 1 x 1 conv as W x; int16 operands only), loaded
      // while the unit's MMAs run
      const int32_t rowb = (CONV && ep.bias_rows && row_ok) ? ep.bias[r] : 0;
      if (!sm100::mbar_wait(tmem_full, i & 1, ep.err, 103, wlim, wstop)) break;
      sm100::tc_fence_after();
      if (ep.partial) {
        for (int cc = R::wc * h; cc < R::wc * h + R::wc; cc += CW) {
          uint32_t hh[CW], mid[CW], ll[CW];
          tmem_ld_cw<CW>(tmem + lane_addr + cc, hh);
          tmem_ld_cw<CW>(tmem + lane_addr + BN + cc, mid);
          tmem_ld_cw<CW>(tmem + lane_addr + 2 * BN + cc, ll);
          sm100::tmem_ld_wait();
          if (cc + CW >= R::wc * h + R::wc) {  // TMEM drained: the next unit's MMAs may start
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(tmem_empty);
          }
          if (!row_ok) continue;
          const uint32_t c0 = w.tile_c + cc;
          // this split's slot of the partial sums ([split][batch][rows][cols])
          unsigned long long* dst = ep.partial +
                                    ((uint64_t)(w.kb0 / ep.kb_per_split) * ep.batch + w.bz) * ep.rows * ep.cols +
                                    (uint64_t)r * ep.cols + c0;
#pragma unroll
          for (int j = 0; j < CW; j++) {
            if (c0 + j >= ep.cols) continue;
            const int64_t acc = ((int64_t)(int32_t)hh[j] << 16) + ((int64_t)(int32_t)mid[j] << 8) + (int64_t)(int32_t)ll[j];
            dst[j] = (unsigned long long)acc;
          }
        }
        continue;
      }
      if (!CONV) {
        // the 64 results of this thread's row as int16 pairs, then TMEM released,
        // then the fused job and the stores
        constexpr int WC = R::wc;
        uint32_t v2[WC / 2];
#pragma unroll
        for (int part = 0; part < WC / CW; part++) {
          const int cc = WC * h + CW * part;
          uint32_t hh[CW], mid[CW], ll[CW];
          tmem_ld_cw<CW>(tmem + lane_addr + cc, hh);
          tmem_ld_cw<CW>(tmem + lane_addr + BN + cc, mid);
          tmem_ld_cw<CW>(tmem + lane_addr + 2 * BN + cc, ll);
          sm100::tmem_ld_wait();
          const uint32_t c0 = w.tile_c + cc;
          combine_any<CW>(ep, hh, mid, ll, c0, v2 + (CW / 2) * part, rowb);
        }
        sm100::tc_fence_before();
        __syncwarp();
        if (lane == 0) sm100::mbar_arrive(tmem_empty);
        if (!row_ok) continue;
        const uint32_t c0 = w.tile_c + WC * h;
        if (ep.mulact) {  // the warp's 32 columns: a gate block, then its up block
          mulact_store(ep, w.bz, r, c0, v2, v2 + 8);
          continue;
        }
        if (ep.post.op != kPostNone) {
          uint32_t b2[WC / 2];
          post_operand<WC>(ep, row_base(ep, w.bz, r), c0, b2);
          post_dispatch<WC / 2>(ep.post, v2, b2);
        }
        store_row<WC>(ep, w.bz, r, c0, v2);
      } else {
        // 16 columns at a time (the register budget of the int16-producer layout):
        // TMEM released after the last chunk's load
        const uint64_t rb = row_ok && ep.post.op != kPostNone ? row_base(ep, w.bz, r) : 0;
        uint32_t g8[8];  // gate / up pairs: the gate block of the pair (even parts)
#pragma unroll 1
        for (int part = 0; part < 4; part++) {
          const int cc = R::wc * h + 16 * part;
          uint32_t hh[16], mid[16], ll[16];
          tmem_ld_cw<16>(tmem + lane_addr + cc, hh);
          tmem_ld_cw<16>(tmem + lane_addr + BN + cc, mid);
          tmem_ld_cw<16>(tmem + lane_addr + 2 * BN + cc, ll);
          sm100::tmem_ld_wait();
          if (part == 3) {
            sm100::tc_fence_before();
            __syncwarp();
            if (lane == 0) sm100::mbar_arrive(tmem_empty);
          }
          if (!row_ok) continue;
          const uint32_t c0 = w.tile_c + cc;
          uint32_t v8[8];
          combine_any<16>(ep, hh, mid, ll, c0, v8, rowb);
          if (ep.mulact) {
            if (part & 1) {
              mulact_store(ep, w.bz, r, c0 - 16, g8, v8);
            } else {
#pragma unroll
              for (int j = 0; j < 8; j++) g8[j] = v8[j];
            }
            continue;
          }
          if (ep.post.op != kPostNone) {
            uint32_t b8[8];
            post_operand<16>(ep, rb, c0, b8);
            post_dispatch<8>(ep.post, v8, b8);
          }
          store_row<16>(ep, w.bz, r, c0, v8);
        }
      }
    }
  }
  sm100::tc_fence_before();
  __syncthreads();
  if (warp == R::mma_warp) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc<TMEM_COLS>(tmem);
  }
}

// K-split units: each split's int64 sums in its own slot (every element of
// every slot written once, no memset, no atomics); this adds them, applies
// the bias and the rule.
__global__ void __launch_bounds__(256) gemm_finish_kernel(const EpiArgs ep) {
  corm_pdl_wait();
  corm_pdl_trigger();
  const uint64_t total = (uint64_t)ep.batch * ep.rows * ep.cols;
  if (ep.mulact) {
    // gate / up pairs (no bias, row-major): output column oc of a row reads
    // gate column 32 (oc / 16) + oc % 16 and the up column 16 after it
    const uint32_t half = ep.cols / 2;
    const uint64_t nout = (uint64_t)ep.batch * ep.rows * half;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nout; i += (uint64_t)gridDim.x * blockDim.x) {
      const uint32_t oc = (uint32_t)(i % half);
      const uint64_t br = i / half;
      const uint32_t r = (uint32_t)(br % ep.rows), bz = (uint32_t)(br / ep.rows);
      const uint64_t cg = br * ep.cols + 32u * (oc / 16u) + oc % 16u;
      unsigned long long sg = 0, su = 0;
      for (uint32_t sp = 0; sp < ep.splits; sp++) {
        sg += __ldg(ep.partial + sp * total + cg);
        su += __ldg(ep.partial + sp * total + cg + 16u);
      }
      const int16_t g = finish((int64_t)sg, ep.flags), u = finish((int64_t)su, ep.flags);
      ep.out[(uint64_t)bz * ep.out_batch_stride + (uint64_t)r * ep.ldc + oc] =
          corm_mulact(g, u, ep.ma_sa, ep.ma_sc, ep.sig);
    }
    return;
  }
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t c = (uint32_t)(i % ep.cols);
    const uint64_t br = i / ep.cols;
    const uint32_t r = (uint32_t)(br % ep.rows), bz = (uint32_t)(br / ep.rows);
    unsigned long long sum = 0;  // the splits' slots in split order (exact integer sums)
    for (uint32_t sp = 0; sp < ep.splits; sp++) sum += __ldg(ep.partial + sp * total + i);
    int64_t acc = (int64_t)sum;
    if (ep.mode == 1 && ep.bias) acc += (int64_t)ep.bias[c] << 8;
    if (ep.bias_rows && ep.bias) acc += (int64_t)ep.bias[r] << 8;
    const uint64_t off = out_offset(ep, ep.mode != 1 ? bz : 0, r, c);
    int16_t y = finish(acc, ep.flags);
    if (ep.post.op != kPostNone) y = post_apply(ep.post, y, post_b(ep.post, off, c));
    ep.out[off] = y;
  }
}

// ---------------------------------------------------------------- split kernels
// dst (b, r, kk) <- src[b*bs + r*ld + kk]; 16 consecutive kk per thread, two
// 16-byte loads when the row is 16-byte aligned, 16-byte stores to each plane.
__device__ __forceinline__ void split16(const SplitSeg& g, uint64_t i) {
  const uint32_t per_row = g.Kp / 16;
  const uint64_t row = i / per_row;  // b * rows + r
  const uint32_t k0 = (uint32_t)(i - row * per_row) * 16;
  const uint64_t b = row / g.rows, r = row - b * g.rows;
  const int16_t* s = g.src + b * g.src_bs + r * g.ld + k0;
  alignas(16) int16_t v[16];
  if (k0 + 16 <= g.K && ((uintptr_t)s & 15) == 0) {
    *(int4*)v = __ldg((const int4*)s);
    *(int4*)(v + 8) = __ldg((const int4*)(s + 8));
  } else {
#pragma unroll
    for (int j = 0; j < 16; j++) v[j] = (k0 + j < g.K) ? __ldg(s + j) : (int16_t)0;
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
  *(int4*)(g.hi + row * g.Kp + k0) = make_int4((int)h[0], (int)h[1], (int)h[2], (int)h[3]);
  *(int4*)(g.lo + row * g.Kp + k0) = make_int4((int)l[0], (int)l[1], (int)l[2], (int)l[3]);
}

__global__ void __launch_bounds__(256) split_rows_kernel(const SplitSeg g, uint64_t total16) {
  corm_pdl_wait();
  corm_pdl_trigger();
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total16; i += (uint64_t)gridDim.x * blockDim.x)
    split16(g, i);
}

__global__ void __launch_bounds__(256) split2_rows_kernel(const SplitSeg ga, uint64_t na, const SplitSeg gb,
                                                          uint64_t nb) {
  corm_pdl_wait();
  corm_pdl_trigger();
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < na + nb; i += (uint64_t)gridDim.x * blockDim.x) {
    if (i < na)
      split16(ga, i);
    else
      split16(gb, i - na);
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

// [planes][outer][inner] bytes, box 128 x 128 x 1, 128-byte swizzle
bool make_map(CUtensorMap* map, const void* base, uint32_t inner, uint32_t outer, uint32_t planes) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {inner, outer, planes};
  cuuint64_t strides[2] = {inner, (cuuint64_t)inner * outer};
  cuuint32_t box[3] = {128, 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// int16 (as 16-bit words) [planes][outer][inner] with row stride ld and plane stride ps
// (elements), box box_inner x box_outer x 1, unswizzled or 128-byte swizzled
// (box_inner 64), zero fill beyond the extents
bool make_raw_map(CUtensorMap* map, const int16_t* base, uint32_t inner, uint32_t outer, uint64_t ld,
                  uint32_t planes, uint64_t ps, uint32_t box_inner, uint32_t box_outer, bool sw128) {
  auto fn = encode_fn();
  if (!fn) return false;
  if (planes <= 1) ps = ld * outer;  // unused extent of one: any valid stride
  cuuint64_t dims[3] = {inner, outer, planes};
  cuuint64_t strides[2] = {ld * 2, ps * 2};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 3, const_cast<int16_t*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct Split {
  uint32_t tiles, num_kb, splits, kps;
};

Split split_of(uint32_t rows, uint32_t cols, uint32_t Kp, uint32_t batch) {
  Split s;
  s.tiles = batch * ((rows + BM - 1) / BM) * ((cols + BN - 1) / BN);
  s.num_kb = (Kp + BK - 1) / BK;
  s.splits = 1;
  // at most half the SMs busy and 12 or more K blocks: split K (at least 4 K
  // blocks per split) to fill the GPU.  A split costs a memset, int64 atomics
  // and a rounding pass over the whole output, which only pay for themselves
  // when the serial K walk is long and the grid is far from full (splitting
  // 8 K blocks, or 128 tiles of K 4096 three ways, measured slower).
  // (Splitting the 8 K blocks of a decode step's 64-row projections too, to
  // one or two blocks a unit, measured slower: 8 layers of the decode step
  // 0.91 ms unsplit, 1.01 to 1.05 ms split 2, 4 or 8 ways.)
  if (s.tiles * 2 <= (uint32_t)NUM_SMS && s.num_kb >= 12) {
    uint32_t want = (2 * NUM_SMS + s.tiles - 1) / s.tiles;
    s.splits = want < s.num_kb / 4 ? want : s.num_kb / 4;
    if (s.splits < 1) s.splits = 1;
  }
  s.kps = (s.num_kb + s.splits - 1) / s.splits;
  s.splits = (s.num_kb + s.kps - 1) / s.kps;
  return s;
}

int* g_err_word[64];
std::mutex g_err_mu;

std::atomic<long long> g_wait_limit{kWaitDefault};

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
  const SplitSeg g{src, src_bs, planes, rows, ld, K, Kp, hi, lo};
  const uint64_t total16 = (uint64_t)planes * rows * (Kp / 16);
  if (total16 == 0) return CORM_OK;
  {
    ProfScope prof_("split_rows_kernel", stream);
    corm_launch_pdl(split_rows_kernel, dim3(corm_blocks(total16, 256, 148u * 16u)), dim3(256), 0, stream, g, total16);
  }
  return cuda_status("split_planes");
}

int split_planes2(const SplitSeg& a, const SplitSeg& b, cudaStream_t stream) {
  const uint64_t na = (uint64_t)a.planes * a.rows * (a.Kp / 16), nb = (uint64_t)b.planes * b.rows * (b.Kp / 16);
  if (na + nb == 0) return CORM_OK;
  {
    ProfScope prof_("split2_rows_kernel", stream);
    corm_launch_pdl(split2_rows_kernel, dim3(corm_blocks(na + nb, 256, 148u * 16u)), dim3(256), 0, stream, a, na, b,
                    nb);
  }
  return cuda_status("split_planes2");
}

size_t gemm_partial_bytes(uint32_t rows, uint32_t cols, uint32_t Kp, uint32_t batch) {
  const Split sp = split_of(rows, cols, Kp, batch);
  return sp.splits > 1 ? (((size_t)sp.splits * batch * rows * cols * 8 + 255) & ~(size_t)255) : 0;
}

int gemm_i8x4(const GemmJob& j, cudaStream_t stream) {
  if (j.Kp % 16 || j.Kp == 0 || j.Kp > kGemmMaxK + 128)
    return fail(CORM_ELIMIT, "gemm: K %u outside 1..%u", j.Kp, kGemmMaxK);
  int* err = j.err ? j.err : device_error_word();
  if (!err) return fail(CORM_ECUDA, "gemm: error word allocation failed");
  CUtensorMap m_ahi, m_alo, m_bhi, m_blo;
  const bool conv = j.a16 != nullptr;  // int16 operands split inside the kernel
  const bool b_planes_in = conv && j.b16 == nullptr;  // A split here, B from its planes
  bool raw_tma = false;
  uint32_t a_box_rows = BM, b_box_cols = BN;
  if (b_planes_in) {
    if ((uintptr_t)j.a16 & 15u || j.lda % 8u || j.a_bs16 % 8u || j.K % 8u || !j.b_hi || !j.b_lo)
      return fail(CORM_EINVAL, "gemm: int16 A not on 16-byte rows, or no B planes");
    memset(&m_alo, 0, sizeof m_alo);
    a_box_rows = j.rows < (uint32_t)BM ? (j.rows + 7u) & ~7u : (uint32_t)BM;
    if (!make_raw_map(&m_ahi, j.a16, j.K, j.rows, j.lda, j.a_bs16 ? j.batch : 1, j.a_bs16, BK / 2, a_box_rows, true) ||
        !make_map(&m_bhi, j.b_hi, j.cols_p, j.K, j.b_planes) || !make_map(&m_blo, j.b_lo, j.cols_p, j.K, j.b_planes))
      return fail(CORM_ECUDA, "gemm: cuTensorMapEncodeTiled failed");
    raw_tma = true;
  } else if (conv) {
    if (((uintptr_t)j.a16 | (uintptr_t)j.b16) & 15u || j.lda % 8u || j.ldb % 8u || j.a_bs16 % 8u || j.b_bs16 % 8u ||
        j.K % 8u || j.cols % 8u)
      return fail(CORM_EINVAL, "gemm: int16 operands not on 16-byte rows");
    memset(&m_ahi, 0, sizeof m_ahi);
    m_alo = m_bhi = m_blo = m_ahi;
    // raw tiles by TMA where both maps encode (A [batch][rows][K], B [batch][K][cols])
    const char* ldg = getenv("CORM_GEMM_LDG_PRODUCERS");  // "1": the plain-load producers instead
    // a job of fewer than 128 rows / columns: boxes that size (multiples of 8)
    a_box_rows = j.rows < (uint32_t)BM ? (j.rows + 7u) & ~7u : (uint32_t)BM;
    b_box_cols = j.cols < (uint32_t)BN ? (j.cols + 7u) & ~7u : (uint32_t)BN;
    raw_tma = !(ldg && ldg[0] == '1') &&
              make_raw_map(&m_ahi, j.a16, j.K, j.rows, j.lda, j.a_bs16 ? j.batch : 1, j.a_bs16, BK / 2, a_box_rows, true) &&
              make_raw_map(&m_bhi, j.b16, j.cols, j.K, j.ldb, j.b_bs16 ? j.batch : 1, j.b_bs16, b_box_cols, BK, false);
  } else {
    bool ok = make_map(&m_ahi, j.a_hi, j.Kp, j.rows, j.a_planes) && make_map(&m_alo, j.a_lo, j.Kp, j.rows, j.a_planes);
    if (j.b_mn)
      ok = ok && make_map(&m_bhi, j.b_hi, j.cols_p, j.K, j.b_planes) && make_map(&m_blo, j.b_lo, j.cols_p, j.K, j.b_planes);
    else
      ok = ok && make_map(&m_bhi, j.b_hi, j.Kp, j.cols, j.b_planes) && make_map(&m_blo, j.b_lo, j.Kp, j.cols, j.b_planes);
    if (!ok) return fail(CORM_ECUDA, "gemm: cuTensorMapEncodeTiled failed");
  }
  const Split sp = split_of(j.rows, j.cols, j.Kp, j.batch);
  EpiArgs ep{};
  ep.mode = j.mode;
  ep.out = j.out;
  if (j.ngroups > 1) {
    // column groups: whole 32-column runs each (the epilogue stores runs of up
    // to 32 columns into one buffer), no fused job, row-major only
    if (j.ngroups > 4 || j.mode != 0 || j.post.op != kPostNone)
      return fail(CORM_EINVAL, "gemm: %u output groups (1..4, row-major, no fused job)", j.ngroups);
    ep.mode = 2;
    uint32_t c = 0;
    for (uint32_t g = 0; g < 4; g++) {
      const bool on = g < j.ngroups;
      if (on && (!j.gout[g] || j.gw[g] == 0 || ((uintptr_t)j.gout[g] & 1u) || (g + 1 < j.ngroups && j.gw[g] % 32u)))
        return fail(CORM_EINVAL, "gemm: output group %u (width %u) not a non-empty run of 32 columns", g, j.gw[g]);
      ep.gc[g] = on ? c : 0xFFFFFFFFu;
      ep.gw[g] = on ? j.gw[g] : 1u;
      ep.gbase[g] = on ? ((int64_t)(intptr_t)j.gout[g] - (int64_t)(intptr_t)j.out) / 2 : 0;
      c += on ? j.gw[g] : 0u;
    }
    ep.gc[4] = 0xFFFFFFFFu;
    if (c != j.cols) return fail(CORM_EINVAL, "gemm: output groups cover %u of %u columns", c, j.cols);
  }
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
  ep.post = j.post;
  {
    const uint32_t kk = j.K ? j.K : j.Kp;
    // int32 when K (2^22 + 2^16 + 2^8) + 2^15 < 2^31; the clamped-HH form
    // while MID + floor(LL / 2^8) + bias < 2^29 (K (2^16 + 2^8) + 2^15)
    ep.ymode = (j.flags & CORM_F_WRAP32) ? 2u
               : ((uint64_t)kk * ((1ull << 22) + (1ull << 16) + (1ull << 8)) + (1ull << 15) < (1ull << 31) ? 0u
                  : ((uint64_t)kk * ((1ull << 16) + (1ull << 8)) + (1ull << 15) < (1ull << 29) ? 1u : 3u));
  }
  if (j.bias_rows && (j.mode != 0 || !j.bias)) return fail(CORM_EINVAL, "gemm: a per-row bias needs mode 0 and a bias");
  ep.bias_rows = j.bias_rows ? 1u : 0u;
  ep.cvar = ((j.flags & CORM_F_ACT_RELU6) ? 6u : ((j.flags & CORM_F_ACT_RELU) ? 3u : 0u)) +
            (j.bias_rows ? 2u : ((j.mode == 1 && j.bias) ? 1u : 0u));
  ep.num_kb = sp.num_kb;
  ep.a_planes = j.a_planes;
  ep.b_planes = j.b_planes;
  ep.b_mn = conv ? 1u : j.b_mn;
  ep.a16 = j.a16;
  ep.b16 = j.b16;
  ep.a_bs16 = j.a_bs16;
  ep.b_bs16 = j.b_bs16;
  ep.lda = j.lda;
  ep.ldb = j.ldb;
  ep.K = j.K ? j.K : j.Kp;
  ep.tiles_m = (j.rows + BM - 1) / BM;
  ep.tiles_n = (j.cols + BN - 1) / BN;
  ep.batch = j.batch;
  ep.splits = sp.splits;
  ep.kb_per_split = sp.kps;
  ep.partial = nullptr;
  ep.err = err;
  ep.wait_limit = g_wait_limit.load(std::memory_order_relaxed);
  ep.raw_tma = raw_tma ? 1u : 0u;
  ep.b_tma_planes = b_planes_in ? 1u : 0u;
  ep.a_box_rows = a_box_rows;
  ep.b_pitch = b_box_cols * 2u;
  ep.m64 = (raw_tma && j.rows <= 64u) ? 1u : 0u;
  if (j.mulact) {
    if (j.mode != 0 || j.ngroups > 1 || j.post.op != kPostNone || j.bias || j.cols % 32u || j.ma_sa < 0 ||
        j.ma_sa > 63 || j.ma_sc < 0 || j.ma_sc > 63)
      return fail(CORM_EINVAL, "gemm: gate / up pairs need one row-major output, no fused job or bias, cols %% 32 == 0");
    const DeviceTables* tb = tables();
    if (!tb) return CORM_ECUDA;
    ep.mulact = 1;
    ep.ma_sa = j.ma_sa;
    ep.ma_sc = j.ma_sc;
    ep.sig = tb->ro_sig;
  }
  if (sp.splits > 1) {
    if (!j.partial) return fail(CORM_ENOMEM, "gemm: K-split job without a partial-sum buffer");
    ep.partial = (unsigned long long*)j.partial;
  }
  static bool attr_set[64];
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_set[dev]) {
    cudaFuncSetAttribute(gemm_i8x4_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(gemm_i8x4_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(gemm_i8x4_kernel<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(gemm_i8x4_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    attr_set[dev] = true;
  }
  const bool diag = ep.wait_limit != kWaitDefault;
  const uint64_t units = (uint64_t)sp.tiles * sp.splits;
  if (units >= (1ull << 31)) return fail(CORM_ELIMIT, "gemm: %llu work units", (unsigned long long)units);
  const unsigned grid = (unsigned)(units < (uint64_t)NUM_SMS ? units : NUM_SMS);
  {
    ProfScope prof_("gemm_i8x4_kernel", stream);
    auto kern = conv ? (diag ? gemm_i8x4_kernel<true, true> : gemm_i8x4_kernel<true, false>)
                     : (diag ? gemm_i8x4_kernel<false, true> : gemm_i8x4_kernel<false, false>);
    const int threads = conv ? Roles<true>::threads : Roles<false>::threads;
    corm_launch_pdl(kern, dim3(grid), dim3(threads), SMEM_BYTES, stream, m_ahi, m_alo, m_bhi, m_blo, ep);
  }
  if (int rc = cuda_status("gemm_i8x4")) return rc;
  if (sp.splits > 1) {
    {
      ProfScope prof_("gemm_finish_kernel", stream);
      const uint64_t nout = (uint64_t)j.batch * j.rows * (j.mulact ? j.cols / 2 : j.cols);
      corm_launch_pdl(gemm_finish_kernel, dim3(corm_blocks(nout, 256)), dim3(256), 0, stream, ep);
    }
    return cuda_status("gemm_finish");
  }
  return CORM_OK;
}

}  // namespace corm

// Reads and clears the per-device word the kernels' bounded waits set on a
// timeout (synchronises the device first), and the word of the allocation-free
// MatMul jobs.  0 = no timeout since the last call.
extern "C" int corm_device_status(int* code) {
  int* w = corm::device_error_word();
  if (!w) return corm::fail(CORM_ECUDA, "corm_device_status: no error word");
  if (cudaDeviceSynchronize() != cudaSuccess) return corm::cuda_status("corm_device_status");
  int v = 0;
  if (cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess) return corm::cuda_status("corm_device_status");
  if (v && cudaMemset(w, 0, sizeof v) != cudaSuccess) return corm::cuda_status("corm_device_status");
  int na = 0;
  if (int rc = corm::noalloc_status_take(&na, nullptr)) return rc;
  if (code) *code = v ? v : na;
  return CORM_OK;
}

// Bounds every mbarrier wait of the GEMM launches that follow (clock cycles;
// <= 0 restores the default of about 2 s).  A diagnostic: limits below 2^20
// cycles read the clock on every probe, so a test can make a wait run out.
extern "C" int corm_set_wait_limit(long long cycles) {
  corm::g_wait_limit.store(cycles > 0 ? cycles : corm::kWaitDefault, std::memory_order_relaxed);
  return CORM_OK;
}
