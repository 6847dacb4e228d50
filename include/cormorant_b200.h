/*
 * cormorant_b200.h — C ABI of the B200 (sm_100a) implementation of the
 * Cormorant fixed-point kernels: VectorOPKernel (with its activation and
 * softmax units), MatmulKernel, ConvKernel, PoolingKernel and RowOpsKernel.
 *
 * Each entry point takes one job descriptor whose fields are the kernel's
 * register block — the same names, units and meaning as the reference's
 * emulated Xilinx drivers (phoenix367/cormorant
 * inference-scheduler/test/host_emu.py) — with DEVICE pointers in place of
 * the physical addresses, plus a CUDA stream.  Calls are stream-ordered and
 * non-blocking (the reference's run_* + kernel_wait pair becomes a launch
 * and a stream synchronise).  Buffers are caller-owned; a job only reads its
 * inputs and writes its output region.
 *
 * Return value: CORM_OK (0), or a negative CORM_E* code for a descriptor the
 * kernel's contract rejects (nothing is launched then) or a CUDA error.
 * corm_last_error() describes the last failure of the calling thread.
 *
 * Element types: int16 storage integers (Q8.8 = ap_fixed<16,8>, or a tensor
 * at a power-of-two exponent); row-ops rows are int16 / int32 / float32 as
 * the op word's kind fields say.
 */
#ifndef CORMORANT_B200_H
#define CORMORANT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* corm_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum {
  CORM_OK = 0,
  CORM_EINVAL = -1,  /* a field outside the kernel's contract */
  CORM_ELIMIT = -2,  /* a size beyond this implementation's limit */
  CORM_ECUDA = -3,   /* a CUDA runtime error (launch, copy, device) */
  CORM_ENOMEM = -4,  /* workspace too small or allocation failed */
  CORM_EDEVICE = -5  /* the current device is not sm_100 */
};

/* Flags shared by MatMul and Conv. */
#define CORM_F_WRAP32 0x1u          /* wrap the exact sum to int32 before the shift (the hardware
                                       accumulator; the simulator's exponent path) */
#define CORM_F_WEIGHT_LOGICAL 0x2u  /* Conv: weight is [out_ch][in_ch | 1][kh][kw], bias [out_ch]
                                       (the simulator's view) instead of the board images */
#define CORM_F_ACT_RELU 0x4u        /* fuse max(y, 0) after the saturation (Conv/MatMul + Relu) */
#define CORM_F_ACT_RELU6 0x8u       /* fuse min(max(y, 0), 6.0) (Clip(0,6)) */

/* ---------------------------------------------------------------- VectorOP
 * Replaces XVectoropkernel_Set_* / XVectoropkernel_Start
 * (inference-scheduler/test/host_emu.py:176-293; kernels/vectorop_rtl/model/
 * include/VectorOP.h:279-333).  c[o*(a_inc+b_inc)+i] = act(op(a[o*a_inc+i],
 * b[o*b_inc+i])) for o < outer, i < size; the last 8-lane word of every
 * output row is written whole with zero tail lanes.  op 0..5 ADD SUB MUL DIV
 * RELU RELU6, 6..9 LEAKY_RELU SILU GELU GELU_TANH, 10/11 softmax row /
 * keys-major column mode (rows at b_inc; smx_cm, smx_cfg = Cs | f_p << 8,
 * smx_mask = valid0 | period << 16).  act 0..6 NONE RELU RELU6 LEAKY_RELU
 * SILU GELU GELU_TANH; LeakyReLU slope alpha[15:0] / 2^16. */
typedef struct {
  const int16_t* a;
  const int16_t* b;  /* unused (may be NULL) for ops 4..11 */
  int16_t* c;
  uint32_t size, op, outer, a_inc, b_inc, act, alpha, smx_cm, smx_cfg, smx_mask;
} corm_vectorop_desc;

int corm_vectorop(const corm_vectorop_desc* d, corm_stream_t stream);

/* ---------------------------------------------------------------- MatMul
 * Replaces XMatmulkernel_Set_* / XMatmulkernel_Start (host_emu.py:312-362;
 * kernels/matmul_rtl/model/include/MatmulKernel.h:195-242).  Per batch slice
 * C[r][j] = sat16(floor(sum_kk A[r][kk] B[kk][j] / 2^8)), A [n][k] and C
 * [n][m] row-major, B row-major [k][m], packed tile-major [ceil(m/32)][k][32]
 * (b_packed) or the GEMV image of width gemv_kw; batch strides in elements,
 * 0 = broadcast.  k <= 4096 (platforms/kv260.json kernels.matmul.max_k).
 * The sum is exact (int64) unless CORM_F_WRAP32.  workspace: device scratch
 * of corm_matmul_workspace_size() bytes (256-byte aligned), or NULL to let the
 * library use its own per-device scratch (grown on demand with cudaMalloc). */
typedef struct {
  const int16_t* a;
  const int16_t* b;
  int16_t* c;
  uint32_t n, k, m, batch, a_batch_stride, b_batch_stride, c_batch_stride, b_packed, gemv_kw;
  uint32_t flags;
  void* workspace;
  size_t workspace_bytes;
} corm_matmul_desc;

int corm_matmul_workspace_size(const corm_matmul_desc* d, size_t* bytes);
int corm_matmul(const corm_matmul_desc* d, corm_stream_t stream);

/* The same MatMul job without any device allocation — no counterpart in the
 * reference.  For callers that must not allocate device memory once running
 * (a generated project whose buffers all come from a pool sized at start-up,
 * or a host whose device memory belongs to another allocator): the job's
 * scratch is a 64 MiB array compiled into the library, which every GPU that
 * loads the library holds until the process exits.  d->workspace is ignored;
 * a job needing more than 64 MiB of scratch returns CORM_ELIMIT.  The first
 * call on a device looks up the array's device address (no allocation); make
 * that first call before any stream capture.  Every call shares the array and
 * it keeps the last call's contents (the job rewrites all it reads), so calls
 * that overlap on the GPU — on different streams, or from several threads —
 * race; serialise them.  Never calls cudaMalloc, cudaFree or any allocating
 * library routine. */
int corm_matmul_noalloc(const corm_matmul_desc* d, corm_stream_t stream);
/* The timeout status of corm_matmul_noalloc jobs, likewise without allocating:
 * waits for the work on `stream` to finish, then reads and clears the word the
 * jobs' bounded waits set when one runs out (*code 0 = none since the last
 * read; a job that ran out left its output incomplete).  Call it when no
 * allocation-free job is in flight on another stream.  corm_device_status
 * reads and clears this word too. */
int corm_matmul_noalloc_status(int* code, corm_stream_t stream);

/* ---------------------------------------------------------------- Conv
 * Replaces XConvkernel_Set_* / XConvkernel_Start (host_emu.py:372-455;
 * kernels/conv_rtl/model/include/ConvKernel.h:229).  y[n][m][oh][ow] =
 * sat16(floor((bias[m] << 8 + sum x w) / 2^8)), x NCHW with zero padding,
 * group 1 or depthwise; weight/bias as the board images (packed tile-major
 * [M][ceil(C/16)][kh][kw][lanes], depthwise [M][roundup(kh*kw,8)], bias
 * word-padded) or logical with CORM_F_WEIGHT_LOGICAL.  Output channel m at
 * (m mod y_cn)*y_cs + (m div y_cn)*y_gs elements (dense when y_cn = y_cs = 0).
 * kh, kw <= 7 and in_ch*kh*kw <= 32768 for group 1 (int32 accumulators stay exact). */
typedef struct {
  const int16_t* x;
  const int16_t* weight;
  const int16_t* bias; /* may be NULL when has_bias == 0 */
  int16_t* y;
  uint32_t batch, in_ch, in_h, in_w, out_ch, out_h, out_w, kh, kw, stride_h, stride_w, dilation_h,
      dilation_w, pad_top, pad_left, has_bias, is_depthwise, y_cs, y_cn, y_gs;
  uint32_t flags;
  void* workspace;
  size_t workspace_bytes;
} corm_conv_desc;

int corm_conv_workspace_size(const corm_conv_desc* d, size_t* bytes);
int corm_conv(const corm_conv_desc* d, corm_stream_t stream);

/* ---------------------------------------------------------------- fused VectorOP epilogue
 * No counterpart in the reference: a MatMul or Conv job followed by a
 * VectorOP job that reads its output, as ONE launch.  The VectorOP job is
 * c = act(op(y, b)) (or op(b, y) with b_is_first) with y the MatMul / Conv
 * result exactly as the plain job writes it and b the second operand:
 * op 0 ADD / 1 SUB -> sat16(x +- z), 2 MUL -> sat16(floor(x z / 2^8)); act is
 * the VectorOP act register (0 none, 1 ReLU, 2 ReLU6, 3 LeakyReLU with alpha,
 * 4 SiLU, 5 GELU, 6 GELU-tanh), the activation unit's rounding included.  b
 * per output column (MatMul) / channel (Conv) — a bias row; at the output's
 * own element offsets — a residual; or one scalar.  The result replaces y in
 * the output buffer (y itself is never stored).  Bit-exact with the two jobs
 * run one after the other. */
enum { CORM_POST_B_COL = 0, CORM_POST_B_SAME = 1, CORM_POST_B_SCALAR = 2 };
typedef struct {
  const int16_t* b;
  uint32_t op;          /* 0 ADD, 1 SUB, 2 MUL */
  uint32_t act, alpha;  /* VectorOP act / alpha registers */
  uint32_t b_mode;      /* CORM_POST_B_* */
  uint32_t b_is_first;  /* SUB: c = b - y */
} corm_postop;

int corm_matmul_post(const corm_matmul_desc* d, const corm_postop* post, corm_stream_t stream);

/* Sibling projections in one launch (no counterpart in the reference): the
 * MatMul job of d (n > 2 rows) with its m output columns split into count
 * (1..4) consecutive groups, group g — width[g] columns, all but the last a
 * multiple of 32 — stored row-major [batch][n][width[g]] at out[g] (batch
 * stride n * width[g]); d->c and d->c_batch_stride are ignored.  Several
 * MatMuls that read the same A and constant weights (q / k / v, gate / up)
 * run as one job over their column-concatenated weights; every output equals
 * its own MatMul's.  Workspace and errors as corm_matmul. */
typedef struct {
  uint32_t count;
  uint32_t width[4];
  int16_t* out[4];
  /* Gate / up pairs (a SwiGLU FFN; no counterpart in the reference): with
   * mulact = 1 and count = 1 the job's m columns (m % 32 == 0) are 16-column
   * blocks alternating gate, up (block 2 i: gate columns 16 i .. 16 i + 15,
   * block 2 i + 1: the up columns of the same outputs), and out[0] (width[0] =
   * m / 2, batch stride n m / 2) receives the row-ops MULACT of each pair with
   * one broadcast entry — sat16(rne(silu_q(g << ma_sa) u / 2^ma_sc)), the
   * unit's SiLU(g) u — instead of the two MatMul outputs.  Equal to the two
   * MatMuls followed by that row-ops job. */
  uint32_t mulact;
  int32_t ma_sa, ma_sc;
} corm_out_groups;
int corm_matmul_groups(const corm_matmul_desc* d, const corm_out_groups* g, corm_stream_t stream);

/* Constant weights split once (no counterpart in the reference): a row-major
 * int16 B [k][m] becomes its int8 hi / lo planes, MN-major [k][mp] with mp =
 * m rounded up to 16 (k * mp bytes each, the padding columns zero). */
int corm_split_b_planes(const int16_t* b, uint32_t k, uint32_t m, int8_t* hi, uint8_t* lo, corm_stream_t stream);
/* The MatMul job of d with B given as those planes (d->b ignored; one B for
 * every batch): the GEMM loads the planes and splits only A, inside the
 * kernel (A on 16-byte rows, k a multiple of 8, n > 2).  g: output column
 * groups as corm_matmul_groups, or NULL for d->c.  The result equals
 * corm_matmul's.  For few rows against a weight read by many jobs (a decode
 * step's projections), where splitting the weight in every job costs most.
 * Workspace: corm_matmul_workspace_size of d suffices. */
int corm_matmul_bplanes(const corm_matmul_desc* d, const int8_t* b_hi, const uint8_t* b_lo, const corm_out_groups* g,
                        corm_stream_t stream);
int corm_conv_post(const corm_conv_desc* d, const corm_postop* post, corm_stream_t stream);

/* ---------------------------------------------------------------- strided batches
 * No counterpart among the reference's kernel registers: what the simulator
 * uses to run the attention of many sequences in one launch.
 *
 * corm_gemm_strided: the MatMul job's numerics (exact int16 sum; CORM_F_WRAP32
 * wraps it to int32; floor / 2^8; sat16; CORM_F_ACT_*) on strided operands:
 * C[b][r][j] at c + b*c_batch_stride + r*ldc + j; A[b][r][kk] at a +
 * b*a_batch_stride + r*lda + kk; B[b][kk][j] at b + b*b_batch_stride +
 * kk*ldb + j, or with b_trans at b + ... + j*ldb + kk.  Strides in elements;
 * a batch stride of 0 shares the operand.  k <= 32768. */
typedef struct {
  const int16_t* a;
  const int16_t* b;
  int16_t* c;
  uint32_t n, k, m, batch;
  uint32_t lda, ldb, ldc, b_trans;
  uint64_t a_batch_stride, b_batch_stride, c_batch_stride;
  uint32_t flags;
  void* workspace; /* NULL: the library's scratch */
  size_t workspace_bytes;
} corm_gemm_desc;

int corm_gemm_strided_workspace_size(const corm_gemm_desc* d, size_t* bytes);
int corm_gemm_strided(const corm_gemm_desc* d, corm_stream_t stream);

/* corm_copy_nd: dst[sum x_i dst_strides[i]] = src[sum x_i src_strides[i]] for
 * every index x over dims[0..ndim) (outermost first, ndim <= 6, strides in
 * int16 elements, may be negative).  The views must not overlap. */
typedef struct {
  const int16_t* src;
  int16_t* dst;
  uint32_t ndim;
  uint32_t dims[6];
  int64_t src_strides[6], dst_strides[6];
} corm_copy_desc;

int corm_copy_nd(const corm_copy_desc* d, corm_stream_t stream);

/* ---------------------------------------------------------------- LLM host operations
 * corm_llm_attn_softmax replaces the host's LlmAttnSoftmax (llm_nodes.py:
 * 1426-1557; C: llm_attn_softmax, llm_nodes.py:2978-3048), the softmax of a
 * decode step: per query column (b G T + h' T + t) of the scores [C][s_stride]
 * the row of P at p + col * p_stride, C entries.  tab: [G][65536] float64,
 * head h' at h' * 65536 (exp(-k 2^-f_s scale), the reference's sexp_table);
 * ip: [G] float64 2^f_p.  n is clamped as the generated code clamps it;
 * window 0: none. */
typedef struct {
  const int16_t* s;
  int16_t* p;
  const double* tab;
  const double* ip;
  uint32_t pos, n, T, G, C, Q, window, batch;
  uint64_t s_stride, p_stride;
} corm_llm_smx_desc;

int corm_llm_attn_softmax(const corm_llm_smx_desc* d, corm_stream_t stream);

/* The float host operations of the LLM entries (llm_nodes.py; the policies
 * that keep the residual stream in float32 on the host), each one launch.
 * Per-channel exponents are int8 arrays on the device; float64 arithmetic in
 * the reference's order with round-to-nearest at every step (no fused
 * multiply-adds); write-back at an exponent = dtype.quantize_exp (RNE,
 * saturated, NaN -> 0).
 *
 * corm_llm_embed replaces LlmEmbed (llm_nodes.py:466-570): out[t][j] =
 * table[clamp(ids[t], 0, rows - 1)][j] (times scale, a float32 product) as
 * float32, or with res32 as the int32 residual RNE(v 2^f). */
typedef struct {
  const int32_t* ids;
  const float* table; /* [rows][d] */
  void* out;          /* float32 or int32 [n][d] */
  uint32_t n, rows, d, res32;
  int32_t f;
  float scale;
} corm_llm_embed_desc;
int corm_llm_embed(const corm_llm_embed_desc* d, corm_stream_t stream);

/* corm_llm_dequant replaces LlmDequant (llm_nodes.py:1722-1750): y =
 * float32(x 2^-f[c]), c = the channel of the last axis (n). */
typedef struct {
  const int16_t* x;
  float* y;
  const int8_t* f; /* [n] */
  uint64_t count;
  uint32_t n;
} corm_llm_dequant_desc;
int corm_llm_dequant(const corm_llm_dequant_desc* d, corm_stream_t stream);

/* corm_llm_resadd replaces LlmResAdd (llm_nodes.py:572-603), the float32
 * residual's add: y = float32((double) h + d 2^-fd[c]). */
typedef struct {
  const float* h;
  const int16_t* d;
  float* y;
  const int8_t* fd; /* [n] */
  uint32_t rows, n;
} corm_llm_resadd_desc;
int corm_llm_resadd(const corm_llm_resadd_desc* d, corm_stream_t stream);

/* corm_llm_rmsnorm replaces LlmRMSNorm (llm_nodes.py:618-694): per row of n,
 * ss = the squares summed left to right, r = 1 / sqrt(ss / n + eps), y =
 * st((h r) gamma[j], fy[c]).  h: float32 rows (h32), or int16 rows of W at
 * per-channel exponents fh[c] (h16; a head norm: every row of W holds W / n
 * rows of n); c = the channel in the row of W; rows counts rows of n. */
typedef struct {
  const float* h32;
  const int16_t* h16;
  const int8_t* fh; /* [W] with h16 */
  int16_t* y;
  const float* gamma; /* [n] */
  const int8_t* fy;   /* [W] */
  double eps;
  uint64_t rows;
  uint32_t n, W;
} corm_llm_rmsnorm_desc;
int corm_llm_rmsnorm(const corm_llm_rmsnorm_desc* d, corm_stream_t stream);

/* corm_llm_act_mul replaces LlmSiluMul / LlmGeluMul (llm_nodes.py:697-791):
 * y = st(T[g_raw + 32768] u 2^-fu[c], fy[c]) with T the float64 activation
 * table (libm exp, built by the caller: silu_table / gelu_table of channel
 * c's gate exponent) at tab + 65536 tab_of[c]. */
typedef struct {
  const int16_t* g;
  const int16_t* u;
  int16_t* y;
  const double* tab;     /* [tables][65536] */
  const uint8_t* tab_of; /* [n] */
  const int8_t* fu;      /* [n] */
  const int8_t* fy;      /* [n] */
  uint32_t rows, n;
} corm_llm_act_mul_desc;
int corm_llm_act_mul(const corm_llm_act_mul_desc* d, corm_stream_t stream);

/* corm_llm_attn_prep_host replaces LlmAttnPrep's host form (llm_nodes.py:
 * 1012-1169) for `batch` sequences at one pos / n: for the rows t < n (n
 * clamped as attn_keys clamps it) RoPE of q0 / k0 in float64 with the float32
 * tables' row pos + t, the K and v rows written into the caches' row pos + t
 * (group-major [KV][batch][C][HD]) at fkc / fvc, and the q.K^T image qx
 * [KV][batch][HD][G T] = clip(RNE(RoPE(q) 2^fq[h])) (columns t >= n: 0).  q0
 * [batch T][ldq] at fq0 [H HD], k0 / v [batch T][ldk / ldv] at fk0 / fv [KV
 * HD]; cos / sin [C][HD / 2] float32. */
typedef struct {
  const int16_t* q0;
  const int16_t* k0;
  const int16_t* v;
  int16_t* kc;
  int16_t* vc;
  int16_t* qx;
  const float* cos;
  const float* sin;
  const int8_t *fq0, *fk0, *fv, *fkc, *fvc, *fq;
  uint32_t pos, n, T, H, KV, HD, C, Q, batch;
  uint64_t ldq, ldk, ldv;
} corm_llm_prep_desc;
int corm_llm_attn_prep_host(const corm_llm_prep_desc* d, corm_stream_t stream);

/* corm_greedy_embed: between two greedy decode steps, per sequence b the
 * next token id = the first index of the largest of logits[b * ld + 0 ..
 * vocab) (int16 at one exponent: LlmDequant then the caller's argmax) and its
 * row of table (int32 [vocab][dim], the embedding as the residual: LlmEmbed,
 * llm_nodes.py:466-560) into out[b * dim ..]; ids (may be NULL) receives the
 * ids. */
typedef struct {
  const int16_t* logits;
  const int32_t* table;
  int32_t* out;
  int32_t* ids;
  uint32_t batch, vocab, dim;
  uint64_t ld;
} corm_greedy_desc;

int corm_greedy_embed(const corm_greedy_desc* d, corm_stream_t stream);

/* corm_llm_decode_attn: one decode step's attention (T = 1) of every KV group
 * of B sequences in one launch — per (sequence b, group g) the q.K^T of the
 * group's G heads over the cache rows the softmax reads (LlmAttnConvNode
 * "qk": exact sum, int32 wrap, floor / 2^8, sat16), the host's p12 softmax
 * (as corm_llm_attn_softmax), the P.V (LlmAttnConvNode "pv") and the head
 * merge (LlmAttnMergeNode): o[b * o_stride + (g G + h') HD + d].  qx: the q
 * image [KV][B][HD][G]; kc / vc: the caches [KV][B][C][HD]; tab: [KV G][65536]
 * float64 per head; ip: [KV G] float64 2^f_p.  G <= 8, HD a divisor of 256. */
typedef struct {
  const int16_t* qx;
  int16_t* kc;
  int16_t* vc;
  const double* tab;
  const double* ip;
  int16_t* o;
  uint32_t pos, B, KV, G, HD, C, Q, window;
  uint64_t o_stride;
  /* The step's AttnPrep fused in (prep bit 0; AttnPrepRoNode with one row,
   * rowops_nodes.py:1112-1143): per sequence b the rows q0 / k0 / v0 at
   * b * ldq / ldk / ldv — RoPE of q0 (entries pq) into the q image (qx is
   * then unused) and of k0 (entries pk) into K cache row pos, v0 re-rounded
   * (entries pv; prep bit 4: copied as is) into V cache row pos; rope: the
   * table [C][2 HD] int32 (cos then sin at 2^-23); prep bits 1 / 2 / 3:
   * pq / pk / pv are one broadcast entry.  The cache rows are written once
   * per (sequence, group), before its scores read them. */
  const int16_t* q0;
  const int16_t* k0;
  const int16_t* v0;
  uint64_t ldq, ldk, ldv;
  const int32_t* rope;
  const void* pq;
  const void* pk;
  const void* pv;
  uint32_t prep;
} corm_llm_decode_attn_desc;

int corm_llm_decode_attn(const corm_llm_decode_attn_desc* d, corm_stream_t stream);

/* ---------------------------------------------------------------- Pool
 * Replaces run_pool / XPoolingkernel (inference-scheduler/src/codegen/
 * _source.py:1548-1580; semantics inference-scheduler/src/codegen/
 * _simulate.py:230-358).  NCHW int16; pool_type 0 MAX, 1 AVG, 2 LP
 * (lp_order 1 or 2); window <= 7x7 except a global window (out 1x1, pool =
 * in). */
typedef struct {
  const int16_t* x;
  int16_t* y;
  uint32_t batch, channels, in_h, in_w, out_h, out_w, pool_h, pool_w, stride_h, stride_w, pad_top,
      pad_left, dil_h, dil_w, pool_type, lp_order, count_include_pad;
} corm_pool_desc;

int corm_pool(const corm_pool_desc* d, corm_stream_t stream);

/* ---------------------------------------------------------------- RowOps
 * Replaces XRowopskernel_Set_* / XRowopskernel_Start (host_emu.py:464-750;
 * kernels/rowops_rtl/tb/verilator/rowops_ref.h:259-427).  op word: [3:0] op
 * (1 COPY, 2 ADDX, 3 DEQUANT, 4 MULACT, 5 NORM, 6 ROPE, 7 XPOSE, 8 TLOAD,
 * 9 FOLD, 10 GATE), [5:4] [7:6] [9:8] A/B/C kinds (0 int16, 1 int32, 2 f32),
 * bit 12 B_EN, 13 P_BCAST, 14 P_KEEP, 15 RELU, 16 NORM_LN, 17 SCALE.  Strides
 * in BYTES; row (i2, i1) of A at a + i2*a_s2 + i1*a_s1.  p: the parameter
 * block, 16 bytes per column.  TLOAD reads the 64 KiB table image from a.
 * n <= 4096. */
typedef struct {
  uint32_t op, n, rows, blocks;
  const void* a;
  uint32_t a_s1, a_s2;
  const void* b;
  uint32_t b_s1, b_s2;
  void* c;
  uint32_t c_s1, c_s2;
  const void* p;
  uint64_t eps;
  uint32_t aux, bq_sh, win_lo, win_hi;
} corm_rowops_desc;

int corm_rowops(const corm_rowops_desc* d, corm_stream_t stream);
/* A descriptor chain (host_emu.py:731-749, rowops_ref.h:428-441): the jobs in
 * order, at most 16, each seeing the writes of the ones before.  Every job
 * (chained or not) keeps the unit's parameter RAM: a job that streams
 * parameters loads it from p unless P_KEEP, and a P_KEEP job reads it.  An
 * ADDX of int32 rows and int16 rows into int32 rows followed by the RMS NORM of
 * its output (a residual add and the next layer's RMSNorm) runs as one pass
 * over the rows, with the same outputs and the same parameter RAM after it. */
int corm_rowops_chain(const corm_rowops_desc* jobs, uint32_t count, corm_stream_t stream);
/* The same with the board's descriptor list in device memory: count 128-byte
 * descriptors at desc, words 0..23 the registers 0x10..0x6C in order (op, n,
 * rows, blocks, a lo / hi, a_s1, a_s2, b lo / hi, b_s1, b_s2, c lo / hi, c_s1,
 * c_s2, p lo / hi, eps lo / hi, aux, bq_sh, win_lo, win_hi).  Reads the list
 * in stream order (a synchronisation of the stream), then runs the chain. */
int corm_rowops_chain_dev(const void* desc, uint32_t count, corm_stream_t stream);

/* ---------------------------------------------------------------- host-side helpers (no GPU) */
/* The activation unit's output for every Q8.8 input (raw -32768 .. 32767 at
 * out[raw + 32768]) — vectorop_act.kernel_table (vectorop_act.py:92-95). */
int corm_act_table(uint32_t act, uint32_t alpha, int16_t* out65536);
/* The softmax unit's TAB[k] = round(2^16 2^(-k/4096)), k < 4096 (vectorop_smx.py:29). */
int corm_smx_table(int32_t* out4096);
/* The 64 KiB OP_TLOAD table image (rowops_spec.table_image, rowops_spec.py:603-616). */
int corm_rowops_table_image(uint8_t* out65536);

/* ---------------------------------------------------------------- device plumbing */
/* Make `device` current for this library's runtime on the calling thread (the
 * library links the CUDA runtime statically; a host that selects devices with
 * its own runtime calls this once per thread). */
int corm_bind_device(int device);
/* Synchronise the current device, then read and clear the status word that the
 * kernels' bounded waits set when a wait times out (0 = none).  Replaces the
 * reference's kernel_wait timeout accounting (runtime/inference_irq.c:259-264). */
int corm_device_status(int* code);
/* Bounds every mbarrier wait of the tensor-core GEMM launches issued after the
 * call, in clock cycles (<= 0 restores the default of about 2 s).  A test and
 * diagnostic knob: below 2^20 cycles the waits read the clock on every probe,
 * so a short limit makes a GEMM's wait run out on purpose; the launch then
 * unwinds and reports through the status words above. */
int corm_set_wait_limit(long long cycles);
/* 1 when every job issued to the stream has finished, 0 while work remains
 * (the drivers' IsDone / IsIdle), or a negative CUDA error. */
int corm_stream_done(corm_stream_t stream);
/* Library version string and the last error message of the calling thread. */
/* Tracing (the analogue of the reference's per-layer profiling aggregates,
 * runtime/inference_prof.h): corm_launch_count() counts every kernel launch of
 * the library; while corm_profile_enable(1) is on, each launch is bracketed by
 * CUDA events on its stream, and corm_profile_read() synchronises, sums them
 * per kernel and clears the record. */
typedef struct {
  char name[48];
  uint64_t launches;
  double total_ms;
  double max_ms;
} corm_profile_entry;
uint64_t corm_launch_count(void);
int corm_profile_enable(int on);
int corm_profile_read(corm_profile_entry* out, int max_entries, int* n_out);

const char* corm_version(void);
const char* corm_last_error(void);

#ifdef __cplusplus
}
#endif
#endif /* CORMORANT_B200_H */
