/*
 * step_from_c.c — a host program in plain C that drives libluma_b200 through
 * its C ABI only (include/luma_b200.h): no Python, no PyTorch.
 *
 * It steps two tensors (an fp32 one and a bf16 one, bf16 grads) twice — the
 * first step, then a quantized step — with the per-step scalars computed in
 * float64 the way the reference's optimizer does (functional.py:262-264;
 * the rows are the same values luma_b200.hostmath.step_row produces), and
 * writes the resulting params, codes and slots to a binary file:
 *
 *   step_from_c <out.bin> <base_seed>
 *
 * Inputs are a fixed integer pattern, reproducible from the test.
 * Build: nvcc -I include step_from_c.c -L luma_b200/_lib -lluma_b200 -lcudart
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "luma_b200.h"

#define N0 70001 /* fp32 params */
#define N1 4099  /* bf16 params */

#define CHECK(call)                                                            \
  do {                                                                         \
    cudaError_t e_ = (call);                                                   \
    if (e_ != cudaSuccess) {                                                   \
      fprintf(stderr, "%s: %s\n", #call, cudaGetErrorString(e_));              \
      return 2;                                                                \
    }                                                                          \
  } while (0)

/* A deterministic value in [-1, 1) from an index (the test recomputes it). */
static float pattern(uint32_t i, uint32_t salt) {
  uint32_t x = i * 2654435761u ^ (salt * 0x9E3779B9u);
  x ^= x >> 15;
  x *= 0x2C1B3C6Du;
  x ^= x >> 12;
  return (float)(x & 0xFFFFFF) / 8388608.0f - 1.0f;
}

static uint16_t to_bf16(float f) { /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static LumaStepRow step_row(int64_t t, double lr, double b1, double b2, double eps, double wd) {
  LumaStepRow r;
  memset(&r, 0, sizeof(r));
  const double bc1 = 1.0 - pow(b1, (double)t), bc2 = 1.0 - pow(b2, (double)t);
  r.step = t;
  r.eps = eps;
  r.beta1 = (float)b1;
  r.omb1 = (float)(1.0 - b1);
  r.beta2 = (float)b2;
  r.omb2 = (float)(1.0 - b2);
  r.decay = (float)(1.0 - wd * lr);
  r.neg_eta = (float)(-(lr / bc1));
  r.inv_bc2 = (float)(1.0 / bc2);
  r.eps32 = (float)eps;
  r.w_max = (float)(1.0 / eps);
  return r;
}

int main(int argc, char** argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: %s <out.bin> <base_seed>\n", argv[0]);
    return 1;
  }
  const int64_t base_seed = strtoll(argv[2], NULL, 10);
  int64_t sizes[5];
  if (luma_abi_version() != LUMA_ABI_VERSION || luma_struct_sizes(sizes, 5) != 5 ||
      sizes[0] != (int64_t)sizeof(LumaTensorDesc) || sizes[4] != (int64_t)sizeof(LumaStepArgs)) {
    fprintf(stderr, "library ABI or struct layout differs from the header\n");
    return 1;
  }

  /* host buffers */
  float* p0 = malloc(N0 * 4);
  uint16_t* p1 = malloc(N1 * 2);
  uint16_t* g0 = malloc(N0 * 2);
  uint16_t* g1 = malloc(N1 * 2);
  for (uint32_t i = 0; i < N0; ++i) p0[i] = 0.02f * pattern(i, 1);
  for (uint32_t i = 0; i < N1; ++i) p1[i] = to_bf16(0.02f * pattern(i, 2));

  /* device buffers (this host may allocate; the library never does) */
  float* d_p0;
  uint16_t *d_p1, *d_g0, *d_g1;
  int16_t *d_qm0, *d_qw0, *d_qm1, *d_qw1;
  LumaTensorDesc* d_desc;
  LumaSlot* d_slots;
  LumaStepRow* d_row;
  CHECK(cudaMalloc((void**)&d_p0, N0 * 4));
  CHECK(cudaMalloc((void**)&d_p1, N1 * 2));
  CHECK(cudaMalloc((void**)&d_g0, N0 * 2));
  CHECK(cudaMalloc((void**)&d_g1, N1 * 2));
  CHECK(cudaMalloc((void**)&d_qm0, N0 * 2));
  CHECK(cudaMalloc((void**)&d_qw0, N0 * 2));
  CHECK(cudaMalloc((void**)&d_qm1, N1 * 2));
  CHECK(cudaMalloc((void**)&d_qw1, N1 * 2));
  CHECK(cudaMalloc((void**)&d_desc, 2 * sizeof(LumaTensorDesc)));
  CHECK(cudaMalloc((void**)&d_slots, 2 * sizeof(LumaSlot)));
  CHECK(cudaMalloc((void**)&d_row, sizeof(LumaStepRow)));
  CHECK(cudaMemset(d_slots, 0, 2 * sizeof(LumaSlot)));
  CHECK(cudaMemcpy(d_p0, p0, N0 * 4, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(d_p1, p1, N1 * 2, cudaMemcpyHostToDevice));

  /* descriptor table: tensor 0 then tensor 1, octets counted from 0 */
  LumaTensorDesc desc[2];
  memset(desc, 0, sizeof(desc));
  desc[0].param = d_p0; desc[0].grad = d_g0; desc[0].q_m = d_qm0; desc[0].q_w = d_qw0;
  desc[0].numel = N0; desc[0].oct_begin = 0; desc[0].param_id = 0; desc[0].slot = 0;
  desc[0].param_dtype = LUMA_F32; desc[0].grad_dtype = LUMA_BF16; desc[0].vec_ok = 1;
  desc[1].param = d_p1; desc[1].grad = d_g1; desc[1].q_m = d_qm1; desc[1].q_w = d_qw1;
  desc[1].numel = N1; desc[1].oct_begin = (N0 + 7) / 8; desc[1].param_id = 1; desc[1].slot = 1;
  desc[1].param_dtype = LUMA_BF16; desc[1].grad_dtype = LUMA_BF16; desc[1].vec_ok = 1;
  CHECK(cudaMemcpy(d_desc, desc, sizeof(desc), cudaMemcpyHostToDevice));

  for (int64_t t = 1; t <= 2; ++t) {
    for (uint32_t i = 0; i < N0; ++i) g0[i] = to_bf16(1e-3f * pattern(i, 10 + (uint32_t)t));
    for (uint32_t i = 0; i < N1; ++i) g1[i] = to_bf16(1e-3f * pattern(i, 20 + (uint32_t)t));
    CHECK(cudaMemcpy(d_g0, g0, N0 * 2, cudaMemcpyHostToDevice));
    CHECK(cudaMemcpy(d_g1, g1, N1 * 2, cudaMemcpyHostToDevice));
    const LumaStepRow row = step_row(t, 1e-3, 0.9, 0.999, 1e-8, 0.01);
    CHECK(cudaMemcpy(d_row, &row, sizeof(row), cudaMemcpyHostToDevice));
    LumaStepArgs a;
    memset(&a, 0, sizeof(a));
    a.descs = d_desc;
    a.slots = d_slots;
    a.rows = d_row;
    a.n_desc = 2;
    a.n_rows = 1;
    a.total_octets = (N0 + 7) / 8 + (N1 + 7) / 8;
    a.base_seed = base_seed;
    if (luma_step(&a, NULL) != LUMA_OK) {
      fprintf(stderr, "luma_step: %s\n", luma_last_error());
      return 3;
    }
    CHECK(cudaDeviceSynchronize());
  }

  /* results: params, codes, slots */
  int16_t* q = malloc(N0 * 2);
  LumaSlot slots[2];
  FILE* f = fopen(argv[1], "wb");
  if (!f) return 4;
  CHECK(cudaMemcpy(p0, d_p0, N0 * 4, cudaMemcpyDeviceToHost));
  fwrite(p0, 4, N0, f);
  CHECK(cudaMemcpy(p1, d_p1, N1 * 2, cudaMemcpyDeviceToHost));
  fwrite(p1, 2, N1, f);
  CHECK(cudaMemcpy(q, d_qm0, N0 * 2, cudaMemcpyDeviceToHost)); fwrite(q, 2, N0, f);
  CHECK(cudaMemcpy(q, d_qw0, N0 * 2, cudaMemcpyDeviceToHost)); fwrite(q, 2, N0, f);
  CHECK(cudaMemcpy(q, d_qm1, N1 * 2, cudaMemcpyDeviceToHost)); fwrite(q, 2, N1, f);
  CHECK(cudaMemcpy(q, d_qw1, N1 * 2, cudaMemcpyDeviceToHost)); fwrite(q, 2, N1, f);
  CHECK(cudaMemcpy(slots, d_slots, sizeof(slots), cudaMemcpyDeviceToHost));
  fwrite(slots, sizeof(slots), 1, f);
  fclose(f);
  printf("ok\n");
  return 0;
}
