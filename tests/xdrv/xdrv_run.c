/*
 * TEST PROGRAM — runs register-level jobs through the Xilinx-style drivers
 * of include/cormorant_b200_xdrv.h (what a generated inference.c calls), on
 * device buffers, and writes the buffers back.  Input file (little-endian):
 *   u32 'XDRV', u32 nbuf, u32 njobs
 *   per buffer: u64 bytes, u8 has_init, [bytes of initial contents]
 *   per job: u32 kind (0 VectorOP, 1 MatMul, 2 Conv, 3 Pool, 4 RowOps, 5 rebase the addresses of a
 *   row-ops descriptor list to device addresses), u32 nregs, u64 regs[nregs]
 * A kind's leading registers are addresses: (buffer index + 1) << 40 | byte
 * offset, 0 for none.  Output file: every buffer's bytes, in order.
 * Exit status 0 when every job was accepted and the device finished.
 */
#define _DEFAULT_SOURCE
#include <stdio.h>
#include <stdlib.h>
#include <unistd.h>

#include <cuda_runtime_api.h>

#include "cormorant_b200_xdrv.h"

static void *g_dev[4096];

static u64 addr(u64 v) {
  if (!v) return 0;
  return (u64)(uintptr_t)g_dev[(v >> 40) - 1] + (v & ((1ull << 40) - 1));
}

int main(int argc, char **argv) {
  if (argc != 3) return 2;
  FILE *f = fopen(argv[1], "rb");
  if (!f) return 2;
  uint32_t hdr[3];
  if (fread(hdr, 4, 3, f) != 3 || hdr[0] != 0x56524458u || hdr[1] > 4096) return 2;
  const uint32_t nbuf = hdr[1], njobs = hdr[2];
  uint64_t *sizes = (uint64_t *)calloc(nbuf, 8);
  if (corm_bind_device(0) != CORM_OK) return 3;
  for (uint32_t i = 0; i < nbuf; i++) {
    uint8_t init;
    if (fread(&sizes[i], 8, 1, f) != 1 || fread(&init, 1, 1, f) != 1) return 2;
    if (cudaMalloc(&g_dev[i], sizes[i] ? sizes[i] : 16) != cudaSuccess) return 3;
    if (init) {
      void *h = malloc(sizes[i]);
      if (fread(h, 1, sizes[i], f) != sizes[i]) return 2;
      cudaMemcpy(g_dev[i], h, sizes[i], cudaMemcpyHostToDevice);
      free(h);
    }
  }
  int bad = 0;
  for (uint32_t j = 0; j < njobs; j++) {
    uint32_t kind, n;
    u64 r[64];
    if (fread(&kind, 4, 1, f) != 1 || fread(&n, 4, 1, f) != 1 || n > 64 || fread(r, 8, n, f) != n) return 2;
    int rc = 0;
    if (kind == 5) {  /* rebase a descriptor list: words 4, 8, 12, 16 (lo / hi) of each 32-word entry */
      uint32_t w[16 * 32];
      void *dd = (void *)(uintptr_t)addr(r[0]);
      const uint32_t nd = (uint32_t)r[1] > 16u ? 16u : (uint32_t)r[1];
      cudaMemcpy(w, dd, 128u * nd, cudaMemcpyDeviceToHost);
      for (uint32_t k = 0; k < nd; k++)
        for (int i = 4; i <= 16; i += 4) {
          const u64 v = addr((u64)w[32 * k + i] | ((u64)w[32 * k + i + 1] << 32));
          w[32 * k + i] = (uint32_t)v;
          w[32 * k + i + 1] = (uint32_t)(v >> 32);
        }
      cudaMemcpy(dd, w, 128u * nd, cudaMemcpyHostToDevice);
      continue;
    }
    if (kind == 0) {
      XVectoropkernel k;
      XVectoropkernel_Initialize(&k, "vectorop");
      XVectoropkernel_Set_a(&k, addr(r[0])); XVectoropkernel_Set_b(&k, addr(r[1])); XVectoropkernel_Set_c(&k, addr(r[2]));
      XVectoropkernel_Set_size(&k, r[3]); XVectoropkernel_Set_op(&k, r[4]); XVectoropkernel_Set_outer(&k, r[5]);
      XVectoropkernel_Set_a_inc(&k, r[6]); XVectoropkernel_Set_b_inc(&k, r[7]); XVectoropkernel_Set_act(&k, r[8]);
      XVectoropkernel_Set_alpha(&k, r[9]); XVectoropkernel_Set_smx_cm(&k, r[10]);
      XVectoropkernel_Set_smx_cfg(&k, r[11]); XVectoropkernel_Set_smx_mask(&k, r[12]);
      XVectoropkernel_Start(&k);
      rc = k.rc;
    } else if (kind == 1) {
      XMatmulkernel k;
      XMatmulkernel_Initialize(&k, "matmul");
      XMatmulkernel_Set_a(&k, addr(r[0])); XMatmulkernel_Set_b(&k, addr(r[1])); XMatmulkernel_Set_c(&k, addr(r[2]));
      XMatmulkernel_Set_n(&k, r[3]); XMatmulkernel_Set_k(&k, r[4]); XMatmulkernel_Set_m(&k, r[5]);
      XMatmulkernel_Set_batch(&k, r[6]); XMatmulkernel_Set_a_batch_stride(&k, r[7]);
      XMatmulkernel_Set_b_batch_stride(&k, r[8]); XMatmulkernel_Set_c_batch_stride(&k, r[9]);
      XMatmulkernel_Set_b_packed(&k, r[10]); XMatmulkernel_Set_gemv_kw(&k, r[11]);
      XMatmulkernel_Start(&k);
      rc = k.rc;
    } else if (kind == 2) {
      XConvkernel k;
      XConvkernel_Initialize(&k, "conv");
      XConvkernel_Set_x(&k, addr(r[0])); XConvkernel_Set_weight(&k, addr(r[1]));
      XConvkernel_Set_bias(&k, addr(r[2])); XConvkernel_Set_y(&k, addr(r[3]));
      XConvkernel_Set_batch(&k, r[4]); XConvkernel_Set_in_ch(&k, r[5]); XConvkernel_Set_in_h(&k, r[6]);
      XConvkernel_Set_in_w(&k, r[7]); XConvkernel_Set_out_ch(&k, r[8]); XConvkernel_Set_out_h(&k, r[9]);
      XConvkernel_Set_out_w(&k, r[10]); XConvkernel_Set_kh(&k, r[11]); XConvkernel_Set_kw(&k, r[12]);
      XConvkernel_Set_stride_h(&k, r[13]); XConvkernel_Set_stride_w(&k, r[14]);
      XConvkernel_Set_dilation_h(&k, r[15]); XConvkernel_Set_dilation_w(&k, r[16]);
      XConvkernel_Set_pad_top(&k, r[17]); XConvkernel_Set_pad_left(&k, r[18]);
      XConvkernel_Set_has_bias(&k, r[19]); XConvkernel_Set_is_depthwise(&k, r[20]);
      XConvkernel_Set_y_cs(&k, r[21]); XConvkernel_Set_y_cn(&k, r[22]); XConvkernel_Set_y_gs(&k, r[23]);
      XConvkernel_Start(&k);
      rc = k.rc;
    } else if (kind == 3) {
      XPoolingkernel k;
      XPoolingkernel_Initialize(&k, "pool");
      XPoolingkernel_Set_x(&k, addr(r[0])); XPoolingkernel_Set_y(&k, addr(r[1]));
      XPoolingkernel_Set_batch(&k, r[2]); XPoolingkernel_Set_channels(&k, r[3]); XPoolingkernel_Set_in_h(&k, r[4]);
      XPoolingkernel_Set_in_w(&k, r[5]); XPoolingkernel_Set_out_h(&k, r[6]); XPoolingkernel_Set_out_w(&k, r[7]);
      XPoolingkernel_Set_pool_h(&k, r[8]); XPoolingkernel_Set_pool_w(&k, r[9]);
      XPoolingkernel_Set_stride_h(&k, r[10]); XPoolingkernel_Set_stride_w(&k, r[11]);
      XPoolingkernel_Set_pad_top(&k, r[12]); XPoolingkernel_Set_pad_left(&k, r[13]);
      XPoolingkernel_Set_dil_h(&k, r[14]); XPoolingkernel_Set_dil_w(&k, r[15]);
      XPoolingkernel_Set_pool_type(&k, r[16]); XPoolingkernel_Set_lp_order(&k, r[17]);
      XPoolingkernel_Set_count_include_pad(&k, r[18]);
      XPoolingkernel_Start(&k);
      rc = k.rc;
    } else {
      XRowopskernel k;
      XRowopskernel_Initialize(&k, "rowops");
      XRowopskernel_Set_a(&k, addr(r[0])); XRowopskernel_Set_b(&k, addr(r[1])); XRowopskernel_Set_c(&k, addr(r[2]));
      XRowopskernel_Set_p(&k, addr(r[3])); XRowopskernel_Set_chain(&k, addr(r[4])); XRowopskernel_Set_eps(&k, r[5]);
      XRowopskernel_Set_op(&k, r[6]); XRowopskernel_Set_n(&k, r[7]); XRowopskernel_Set_rows(&k, r[8]);
      XRowopskernel_Set_blocks(&k, r[9]); XRowopskernel_Set_a_s1(&k, r[10]); XRowopskernel_Set_a_s2(&k, r[11]);
      XRowopskernel_Set_b_s1(&k, r[12]); XRowopskernel_Set_b_s2(&k, r[13]); XRowopskernel_Set_c_s1(&k, r[14]);
      XRowopskernel_Set_c_s2(&k, r[15]); XRowopskernel_Set_aux(&k, r[16]); XRowopskernel_Set_bq_sh(&k, r[17]);
      XRowopskernel_Set_win_lo(&k, r[18]); XRowopskernel_Set_win_hi(&k, r[19]); XRowopskernel_Set_chain_n(&k, r[20]);
      XRowopskernel_Start(&k);
      rc = k.rc;
    }
    if (rc != CORM_OK) {
      fprintf(stderr, "job %u (kind %u): rc %d: %s\n", j, kind, rc, corm_last_error());
      bad = 1;
    }
  }
  /* the drivers' completion poll, bounded */
  int done = 0;
  for (int it = 0; it < 200000 && !done; it++) {
    done = corm_xdrv_done();
    if (!done) usleep(50);
  }
  if (!done) {
    fprintf(stderr, "device did not finish\n");
    return 4;
  }
  FILE *o = fopen(argv[2], "wb");
  for (uint32_t i = 0; i < nbuf; i++) {
    void *h = malloc(sizes[i] ? sizes[i] : 1);
    cudaMemcpy(h, g_dev[i], sizes[i], cudaMemcpyDeviceToHost);
    fwrite(h, 1, sizes[i], o);
    free(h);
    cudaFree(g_dev[i]);
  }
  fclose(o);
  return bad;
}
