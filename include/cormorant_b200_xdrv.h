/*
 * cormorant_b200_xdrv.h — the Xilinx-style kernel drivers the generated
 * inference projects call (XVectoropkernel_*, XMatmulkernel_*,
 * XConvkernel_*, XPoolingkernel_*, XRowopskernel_*: the register setters,
 * Start, IsDone / IsIdle, Release), implemented over the cormorant_b200 C ABI
 * so that a generated inference.c runs unchanged on a B200.  Same structs,
 * register names and field semantics as the reference's software models of
 * the drivers (phoenix367/cormorant inference-scheduler/test/host_emu.py:
 * 162-750); the "physical addresses" a project programs are device
 * addresses here (its inference_buf_phys returns the device pointer).
 *
 * Start issues the job on the driver stream (corm_xdrv_stream, NULL = the
 * legacy default stream; set it per thread with corm_xdrv_set_stream) and
 * returns at once, as the board's kernels do; IsDone / IsIdle report whether
 * that stream has finished.  The job's return code (CORM_OK or a CORM_E*
 * code for a register block the kernel's contract rejects) is kept in the
 * struct's `rc`.  The layouts the board uses are the ones these take: packed
 * / GEMV-image B (b_packed, gemv_kw), the tile-major conv weight image, the
 * y channel pattern, descriptor chains read from device memory.  The GEMV
 * register a_to_b has no effect (the B200 GEMV reads A directly).
 *
 * Header-only C99; link with libcorm_b200.so.
 */
#ifndef CORMORANT_B200_XDRV_H
#define CORMORANT_B200_XDRV_H

#include <stdint.h>
#include <string.h>

#include "cormorant_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef uint64_t u64;

static corm_stream_t corm_xdrv_stream = 0;
static inline void corm_xdrv_set_stream(corm_stream_t s) { corm_xdrv_stream = s; }
static inline int corm_xdrv_done(void) { return corm_stream_done(corm_xdrv_stream) == 1; }

#define CORM_XDRV_PTR(v) ((void *)(uintptr_t)(v))

/* ---------------------------------------------------------------- VectorOP (host_emu.py:176-306) */
#define XVECTOROPKERNEL_CTRL_ADDR_ALPHA_DATA 0x64
#define XVECTOROPKERNEL_CTRL_ADDR_SMX_CM_DATA 0x6c
typedef struct {
  u64 Ctrl_BaseAddress;
  u64 a, b, c;
  uint32_t size, op, outer, a_inc, b_inc, act, alpha, smx_cm, smx_cfg, smx_mask;
  int rc;
} XVectoropkernel;
static inline int XVectoropkernel_Initialize(XVectoropkernel *p, const char *n) {
  (void)n;
  memset(p, 0, sizeof *p);
  return 0;
}
static inline void XVectoropkernel_Set_a(XVectoropkernel *p, u64 v) { p->a = v; }
static inline void XVectoropkernel_Set_b(XVectoropkernel *p, u64 v) { p->b = v; }
static inline void XVectoropkernel_Set_c(XVectoropkernel *p, u64 v) { p->c = v; }
#define CORM_VOP_SET(f) \
  static inline void XVectoropkernel_Set_##f(XVectoropkernel *p, u64 v) { p->f = (uint32_t)v; }
CORM_VOP_SET(size) CORM_VOP_SET(op) CORM_VOP_SET(outer) CORM_VOP_SET(a_inc) CORM_VOP_SET(b_inc)
CORM_VOP_SET(act) CORM_VOP_SET(alpha) CORM_VOP_SET(smx_cm) CORM_VOP_SET(smx_cfg) CORM_VOP_SET(smx_mask)
static inline uint32_t XVectoropkernel_Get_alpha(XVectoropkernel *p) { return p->alpha; }
static inline uint32_t XVectoropkernel_Get_smx_cm(XVectoropkernel *p) { return p->smx_cm; }
static inline void XVectoropkernel_Start(XVectoropkernel *p) {
  corm_vectorop_desc d;
  memset(&d, 0, sizeof d);
  d.a = (const int16_t *)CORM_XDRV_PTR(p->a);
  d.b = (const int16_t *)CORM_XDRV_PTR(p->b);
  d.c = (int16_t *)CORM_XDRV_PTR(p->c);
  d.size = p->size; d.op = p->op; d.outer = p->outer; d.a_inc = p->a_inc; d.b_inc = p->b_inc;
  d.act = p->act; d.alpha = p->alpha; d.smx_cm = p->smx_cm; d.smx_cfg = p->smx_cfg; d.smx_mask = p->smx_mask;
  p->rc = corm_vectorop(&d, corm_xdrv_stream);
}
static inline int XVectoropkernel_IsDone(XVectoropkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XVectoropkernel_IsIdle(XVectoropkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XVectoropkernel_Release(XVectoropkernel *p) { (void)p; return 0; }

/* ---------------------------------------------------------------- MatMul (host_emu.py:312-362) */
typedef struct {
  u64 Ctrl_BaseAddress;
  u64 a, b, c, a_to_b;
  uint32_t n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, b_packed, gemv_kw;
  int rc;
} XMatmulkernel;
static inline int XMatmulkernel_Initialize(XMatmulkernel *p, const char *n) {
  (void)n;
  memset(p, 0, sizeof *p);
  return 0;
}
static inline void XMatmulkernel_Set_a(XMatmulkernel *p, u64 v) { p->a = v; }
static inline void XMatmulkernel_Set_b(XMatmulkernel *p, u64 v) { p->b = v; }
static inline void XMatmulkernel_Set_c(XMatmulkernel *p, u64 v) { p->c = v; }
static inline void XMatmulkernel_Set_a_to_b(XMatmulkernel *p, u64 v) { p->a_to_b = v; }
#define CORM_MM_SET(f) \
  static inline void XMatmulkernel_Set_##f(XMatmulkernel *p, u64 v) { p->f = (uint32_t)v; }
CORM_MM_SET(n) CORM_MM_SET(k) CORM_MM_SET(m) CORM_MM_SET(batch) CORM_MM_SET(a_batch_stride)
CORM_MM_SET(b_batch_stride) CORM_MM_SET(c_batch_stride) CORM_MM_SET(b_packed) CORM_MM_SET(gemv_kw)
static inline void XMatmulkernel_Start(XMatmulkernel *p) {
  corm_matmul_desc d;
  memset(&d, 0, sizeof d);
  d.a = (const int16_t *)CORM_XDRV_PTR(p->a);
  d.b = (const int16_t *)CORM_XDRV_PTR(p->b);
  d.c = (int16_t *)CORM_XDRV_PTR(p->c);
  d.n = p->n; d.k = p->k; d.m = p->m; d.batch = p->batch ? p->batch : 1u;
  d.a_batch_stride = p->a_batch_stride; d.b_batch_stride = p->b_batch_stride; d.c_batch_stride = p->c_batch_stride;
  d.b_packed = p->b_packed; d.gemv_kw = p->gemv_kw;
  p->rc = corm_matmul(&d, corm_xdrv_stream);
}
static inline int XMatmulkernel_IsDone(XMatmulkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XMatmulkernel_IsIdle(XMatmulkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XMatmulkernel_Release(XMatmulkernel *p) { (void)p; return 0; }

/* ---------------------------------------------------------------- Conv (host_emu.py:366-455) */
#define XCONVKERNEL_CTRL_ADDR_Y_CS_DATA 0xc8
typedef struct {
  u64 Ctrl_BaseAddress;
  u64 x, weight, bias, y;
  uint32_t batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h, dilation_w,
      pad_top, pad_left, has_bias, is_depthwise, y_cs, y_cn, y_gs;
  int rc;
} XConvkernel;
static inline int XConvkernel_Initialize(XConvkernel *p, const char *n) {
  (void)n;
  memset(p, 0, sizeof *p);
  return 0;
}
static inline void XConvkernel_Set_x(XConvkernel *p, u64 v) { p->x = v; }
static inline void XConvkernel_Set_weight(XConvkernel *p, u64 v) { p->weight = v; }
static inline void XConvkernel_Set_bias(XConvkernel *p, u64 v) { p->bias = v; }
static inline void XConvkernel_Set_y(XConvkernel *p, u64 v) { p->y = v; }
#define CORM_CV_SET(f) \
  static inline void XConvkernel_Set_##f(XConvkernel *p, u64 v) { p->f = (uint32_t)v; }
CORM_CV_SET(batch) CORM_CV_SET(in_ch) CORM_CV_SET(in_h) CORM_CV_SET(in_w) CORM_CV_SET(out_ch)
CORM_CV_SET(out_h) CORM_CV_SET(out_w) CORM_CV_SET(kh) CORM_CV_SET(kw) CORM_CV_SET(stride_h)
CORM_CV_SET(stride_w) CORM_CV_SET(dilation_h) CORM_CV_SET(dilation_w) CORM_CV_SET(pad_top)
CORM_CV_SET(pad_left) CORM_CV_SET(has_bias) CORM_CV_SET(is_depthwise) CORM_CV_SET(y_cs)
CORM_CV_SET(y_cn) CORM_CV_SET(y_gs)
static inline void XConvkernel_Start(XConvkernel *p) {
  corm_conv_desc d;
  memset(&d, 0, sizeof d);
  d.x = (const int16_t *)CORM_XDRV_PTR(p->x);
  d.weight = (const int16_t *)CORM_XDRV_PTR(p->weight);
  d.bias = (const int16_t *)CORM_XDRV_PTR(p->bias);
  d.y = (int16_t *)CORM_XDRV_PTR(p->y);
  d.batch = p->batch; d.in_ch = p->in_ch; d.in_h = p->in_h; d.in_w = p->in_w; d.out_ch = p->out_ch;
  d.out_h = p->out_h; d.out_w = p->out_w; d.kh = p->kh; d.kw = p->kw; d.stride_h = p->stride_h;
  d.stride_w = p->stride_w; d.dilation_h = p->dilation_h; d.dilation_w = p->dilation_w; d.pad_top = p->pad_top;
  d.pad_left = p->pad_left; d.has_bias = p->has_bias; d.is_depthwise = p->is_depthwise; d.y_cs = p->y_cs;
  d.y_cn = p->y_cn; d.y_gs = p->y_gs;
  d.flags = 0; /* the board's tile-major weight image */
  p->rc = corm_conv(&d, corm_xdrv_stream);
}
static inline int XConvkernel_IsDone(XConvkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XConvkernel_IsIdle(XConvkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XConvkernel_Release(XConvkernel *p) { (void)p; return 0; }

/* ---------------------------------------------------------------- Pool (codegen/_source.py:1548-1580) */
typedef struct {
  u64 Ctrl_BaseAddress;
  u64 x, y;
  uint32_t batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top, pad_left, dil_h,
      dil_w, pool_type, lp_order, count_include_pad;
  int rc;
} XPoolingkernel;
static inline int XPoolingkernel_Initialize(XPoolingkernel *p, const char *n) {
  (void)n;
  memset(p, 0, sizeof *p);
  return 0;
}
static inline void XPoolingkernel_Set_x(XPoolingkernel *p, u64 v) { p->x = v; }
static inline void XPoolingkernel_Set_y(XPoolingkernel *p, u64 v) { p->y = v; }
#define CORM_PL_SET(f) \
  static inline void XPoolingkernel_Set_##f(XPoolingkernel *p, u64 v) { p->f = (uint32_t)v; }
CORM_PL_SET(batch) CORM_PL_SET(channels) CORM_PL_SET(in_h) CORM_PL_SET(in_w) CORM_PL_SET(out_h)
CORM_PL_SET(out_w) CORM_PL_SET(pool_h) CORM_PL_SET(pool_w) CORM_PL_SET(stride_h) CORM_PL_SET(stride_w)
CORM_PL_SET(pad_top) CORM_PL_SET(pad_left) CORM_PL_SET(dil_h) CORM_PL_SET(dil_w) CORM_PL_SET(pool_type)
CORM_PL_SET(lp_order) CORM_PL_SET(count_include_pad)
static inline void XPoolingkernel_Start(XPoolingkernel *p) {
  corm_pool_desc d;
  memset(&d, 0, sizeof d);
  d.x = (const int16_t *)CORM_XDRV_PTR(p->x);
  d.y = (int16_t *)CORM_XDRV_PTR(p->y);
  d.batch = p->batch; d.channels = p->channels; d.in_h = p->in_h; d.in_w = p->in_w; d.out_h = p->out_h;
  d.out_w = p->out_w; d.pool_h = p->pool_h; d.pool_w = p->pool_w; d.stride_h = p->stride_h;
  d.stride_w = p->stride_w; d.pad_top = p->pad_top; d.pad_left = p->pad_left; d.dil_h = p->dil_h;
  d.dil_w = p->dil_w; d.pool_type = p->pool_type; d.lp_order = p->lp_order;
  d.count_include_pad = p->count_include_pad;
  p->rc = corm_pool(&d, corm_xdrv_stream);
}
static inline int XPoolingkernel_IsDone(XPoolingkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XPoolingkernel_IsIdle(XPoolingkernel *p) { (void)p; return corm_xdrv_done(); }
static inline int XPoolingkernel_Release(XPoolingkernel *p) { (void)p; return 0; }

/* ---------------------------------------------------------------- RowOps (host_emu.py:460-750) */
#define XROWOPSKERNEL_CTRL_ADDR_CHAIN_N_DATA 0x78
typedef struct {
  u64 Ctrl_BaseAddress;
  u64 a, b, c, p, eps;
  uint32_t op, n, rows, blocks, a_s1, a_s2, b_s1, b_s2, c_s1, c_s2, aux, bq_sh, win_lo, win_hi;
  u64 chain;
  uint32_t chain_n;
  int rc;
} XRowopskernel;
static inline int XRowopskernel_Initialize(XRowopskernel *q, const char *nm) {
  (void)nm;
  memset(q, 0, sizeof *q);
  return 0;
}
#define CORM_RO_SET(f) \
  static inline void XRowopskernel_Set_##f(XRowopskernel *q, u64 v) { q->f = (uint32_t)v; }
static inline void XRowopskernel_Set_a(XRowopskernel *q, u64 v) { q->a = v; }
static inline void XRowopskernel_Set_b(XRowopskernel *q, u64 v) { q->b = v; }
static inline void XRowopskernel_Set_c(XRowopskernel *q, u64 v) { q->c = v; }
static inline void XRowopskernel_Set_p(XRowopskernel *q, u64 v) { q->p = v; }
static inline void XRowopskernel_Set_eps(XRowopskernel *q, u64 v) { q->eps = v; }
CORM_RO_SET(op) CORM_RO_SET(n) CORM_RO_SET(rows) CORM_RO_SET(blocks) CORM_RO_SET(a_s1) CORM_RO_SET(a_s2)
CORM_RO_SET(b_s1) CORM_RO_SET(b_s2) CORM_RO_SET(c_s1) CORM_RO_SET(c_s2) CORM_RO_SET(aux) CORM_RO_SET(bq_sh)
CORM_RO_SET(win_lo) CORM_RO_SET(win_hi) CORM_RO_SET(chain_n)
static inline void XRowopskernel_Set_chain(XRowopskernel *q, u64 v) { q->chain = v; }
/* Start: one job from the registers, or (chain_n != 0) the 128-byte
 * descriptors at device address chain — words 0..23 the registers 0x10..0x6C
 * in order, at most 16 (host_emu.py:731-749). */
static inline void XRowopskernel_Start(XRowopskernel *q) {
  if (q->chain_n) {
    q->rc = corm_rowops_chain_dev(CORM_XDRV_PTR(q->chain), q->chain_n, corm_xdrv_stream);
    return;
  }
  corm_rowops_desc d;
  memset(&d, 0, sizeof d);
  d.op = q->op; d.n = q->n; d.rows = q->rows; d.blocks = q->blocks;
  d.a = CORM_XDRV_PTR(q->a); d.a_s1 = q->a_s1; d.a_s2 = q->a_s2;
  d.b = CORM_XDRV_PTR(q->b); d.b_s1 = q->b_s1; d.b_s2 = q->b_s2;
  d.c = CORM_XDRV_PTR(q->c); d.c_s1 = q->c_s1; d.c_s2 = q->c_s2;
  d.p = CORM_XDRV_PTR(q->p); d.eps = q->eps; d.aux = q->aux; d.bq_sh = q->bq_sh;
  d.win_lo = q->win_lo; d.win_hi = q->win_hi;
  q->rc = corm_rowops(&d, corm_xdrv_stream);
}
static inline int XRowopskernel_IsDone(XRowopskernel *q) { (void)q; return corm_xdrv_done(); }
static inline int XRowopskernel_IsIdle(XRowopskernel *q) { (void)q; return corm_xdrv_done(); }
static inline int XRowopskernel_Release(XRowopskernel *q) { (void)q; return 0; }

#ifdef __cplusplus
}
#endif
#endif /* CORMORANT_B200_XDRV_H */
