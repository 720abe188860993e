/*
 * luma_b200.h — C ABI of the B200 (sm_100a) LUMA optimizer step.
 *
 * LUMA keeps AdamW's two moments as int16 codes on a per-tensor logarithmic
 * grid (Q_m: signed momentum codes, Q_w: unsigned preconditioner codes stored
 * in int16 bits) with per-tensor scales S_m = max|m|, S_v = max v.  One step
 * decodes the codes, forms the new EMAs, applies the decoupled-weight-decay
 * AdamW update, finds the new scales and re-quantizes onto the grid those
 * scales define, with unbiased log-to-linear stochastic rounding (LogSR).
 *
 * This library runs that step for many tensors at once as two kernel
 * launches over a device-resident descriptor table:
 *   pass 1: decode -> EMA -> per-tensor max|m'|, max v'  (the last CTA to
 *           finish a tensor turns the maxima into the next log grid);
 *   pass 2: decode -> EMA -> AdamW update of the param (fp32 or bf16, in
 *           place) -> LogSR re-quantization of m', v' (int16, in place).
 *
 * Every entry point is plain C: raw device pointers, sizes and a CUDA stream
 * handle (cudaStream_t passed as void*).  Nothing here allocates device
 * memory; the caller owns every buffer.  Calls are asynchronous on `stream`
 * and return a status code (LUMA_OK on success; luma_last_error() gives the
 * message of the last failure on the calling thread).
 *
 * Reference interfaces replaced (IgorYashch/LUMA, src/luma_optimizer/):
 *   luma_step  <- triton_kernel.py:449-492  luma_triton_step(...)
 *                 triton_kernel.py:409-446  luma_triton_init_step(...)
 *                 functional.py:231-298     luma_update_step(...)
 *                 functional.py:183-228     luma_init_step(...)
 *              (one call steps every tensor whose descriptor is in the
 *               table; the reference calls one of those per tensor from the
 *               per-parameter loop at optimizer.py:422-522)
 *   LumaGrid   <- functional.py:74-92 _precompute(S_m, S_v, eps) outputs,
 *                 triton_kernel.py:34-36 new_grid[8] buffer layout
 *   LumaStepRow<- functional.py:262-264 host scalars (bc1, bc2, eta_t) and
 *                 optimizer.py:423-426 per-group hyper-parameters
 */
#ifndef LUMA_B200_H
#define LUMA_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LUMA_ABI_VERSION 4

/* Quantization grid constants (reference config.py:23-25). */
#define LUMA_K_M 32767        /* signed int16 magnitude of Q_m        */
#define LUMA_K_W 65535        /* unsigned 16-bit range of Q_w         */
#define LUMA_SCALE_FLOOR_M 1e-9

/* Element types of params and grads. */
enum {
  LUMA_F32 = 0,
  LUMA_BF16 = 1,
  LUMA_F16 = 2
};

/* Status codes. */
enum {
  LUMA_OK = 0,
  LUMA_ERR_INVALID = 1,     /* bad argument: null pointer, bad dtype, size */
  LUMA_ERR_CUDA = 2,        /* a CUDA runtime call failed                 */
  LUMA_ERR_UNSUPPORTED = 3  /* current device is not sm_100               */
};

/*
 * One tensor (or one shard segment of a tensor) to step.  Device pointers.
 * The table handed to luma_step must be sorted by oct_begin, with
 * oct_begin[i+1] == oct_begin[i] + ceil(numel[i] / 8): the flat work space is
 * counted in octets (groups of 8 elements) so every split point is 8-aligned.
 */
typedef struct LumaTensorDesc {
  void*        param;        /* fp32 or bf16 [numel], updated in place      */
  const void*  grad;         /* fp32, bf16 or fp16 [numel]                  */
  int16_t*     q_m;          /* int16 [numel] momentum codes, in place      */
  int16_t*     q_w;          /* int16 [numel] preconditioner codes (uint16
                                bits), in place                             */
  const float* u_m;          /* test hook: injected uniforms for Q_m, or NULL
                                for the Philox4x32-10 stream                */
  const float* u_w;          /* test hook: injected uniforms for Q_w, or NULL */
  int64_t      numel;        /* elements (>= 1)                             */
  int64_t      oct_begin;    /* first octet of this tensor in the flat space */
  int64_t      rng_offset;   /* Philox counter of element 0 (multiple of 8);
                                a shard segment passes its offset inside the
                                full tensor                                 */
  int32_t      param_id;     /* reference parameter index (seed mixing)     */
  int32_t      row;          /* index into the LumaStepRow table            */
  int32_t      slot;         /* index into the LumaSlot state array         */
  uint8_t      param_dtype;  /* LUMA_F32 | LUMA_BF16                        */
  uint8_t      grad_dtype;   /* LUMA_F32 | LUMA_BF16 | LUMA_F16             */
  uint8_t      vec_ok;       /* 1 if param/grad/q_m/q_w/u_m/u_w are 16-byte
                                aligned (128-bit vector path)               */
  uint8_t      mc_local;     /* with param_mc: 1 if pass 2 also stores the
                                updated param to `param` (param_mc then maps a
                                different buffer, e.g. the staging buffer of a
                                sharded-params gather); 0 if param_mc maps
                                `param` itself                              */
  void*        param_mc;     /* NULL, or an NVLink multicast (NVLS) address:
                                pass 2 writes the updated param through it
                                with multimem stores, so every GPU bound to
                                the multicast object gets it in the same step
                                (the ZeRO all-gather fused into the step).
                                When it maps `param` itself (mc_local = 0) the
                                local copy arrives the same way.  Requires
                                param and param_mc 8-byte
                                aligned and, for an odd numel of bf16 params,
                                that the 2 bytes after the last element belong
                                to the caller (they are written: multimem
                                stores are 32 bits wide at least).  The caller
                                orders these writes against other readers of
                                the peers' copies (a barrier before and after
                                the step).                                   */
} LumaTensorDesc;            /* 96 bytes */

/*
 * Per-step scalars of one (param group, step) class, computed on the host in
 * float64 exactly as the reference does and rounded to float32 where the
 * reference's tensor ops round a Python scalar (functional.py:259-279).
 */
typedef struct LumaStepRow {
  int64_t step;      /* t after the increment (optimizer.py:457); 1 = first step */
  double  eps;       /* group eps, float64 (grid precompute)                */
  float   beta1;     /* fl32(beta1)                                          */
  float   omb1;      /* fl32(1 - beta1)                                      */
  float   beta2;     /* fl32(beta2)                                          */
  float   omb2;      /* fl32(1 - beta2)                                      */
  float   decay;     /* fl32(1 - weight_decay * lr)                          */
  float   neg_eta;   /* fl32(-(lr / (1 - beta1^t)))                          */
  float   inv_bc2;   /* fl32(1.0 / (1 - beta2^t)), float64 reciprocal       */
  float   eps32;     /* fl32(eps)                                            */
  float   w_max;     /* fl32(1 / eps)                                        */
  float   reserved;
} LumaStepRow;       /* 56 bytes */

/*
 * One log grid (functional.py:74-92 evaluated for (S_m, S_v, eps)), with the
 * float32 values the element-wise code consumes.  A reference expression
 * "tensor / s" with a Python float s is evaluated on CUDA as
 * tensor * fl32(1.0 / s) (reciprocal in float64), hence the inv_* fields.
 */
typedef struct LumaGrid {
  double  S_m;       /* max(max|m|, 1e-9), as the reference stores it       */
  double  S_v;       /* max(max v, 0)                                        */
  double  eps;       /* eps the float32 fields below were derived with      */
  float   dm;        /* fl32(delta_m)                                        */
  float   inv_dm;    /* fl32(1.0 / delta_m)                                */
  float   inv_zm;    /* fl32(1.0 / z_m)                                      */
  float   s_m32;     /* fl32(S_m) (momentum clamp)                           */
  float   w_min;     /* fl32(w_min)                                          */
  float   inv_wmin;  /* fl32(1.0 / w_min)                                    */
  float   dw;        /* fl32(delta_w)                                        */
  float   inv_dw;    /* fl32(1.0 / delta_w), 0 when delta_w == 0             */
  float   inv_zw;    /* fl32(1.0 / z_w)                                      */
  int32_t dw_pos;    /* delta_w > 0                                          */
} LumaGrid;          /* 64 bytes */

/*
 * Device state of one descriptor.  grid[t & 1] holds the grid the codes were
 * written on at step t; step t decodes with grid[(t - 1) & 1] and encodes
 * with grid[t & 1].  amax_m/amax_v/done are pass-1 accumulators: zero before
 * a step, reset to zero by the CTA that finishes the tensor.  A new slot must
 * be zero-filled.
 */
typedef struct LumaSlot {
  LumaGrid grid[2];
  uint32_t amax_m;   /* bits of max |m'| (non-negative float order)         */
  uint32_t amax_v;   /* bits of max v'                                       */
  uint64_t done;     /* octets of this tensor finished by pass 1            */
} LumaSlot;          /* 144 bytes */

typedef struct LumaStepArgs {
  const LumaTensorDesc* descs;    /* device [n_desc], sorted by oct_begin   */
  LumaSlot*             slots;    /* device state array                     */
  const LumaStepRow*    rows;     /* device [n_rows]                        */
  int32_t               n_desc;
  int32_t               n_rows;
  int64_t               total_octets; /* oct_begin[last] + octets(last)     */
  int64_t               base_seed;    /* optimizer._base_seed (optimizer.py:94-96) */
  void*                 events[3];    /* optional cudaEvent_t recorded before
                                         pass 1, between the passes and after
                                         pass 2 (timing); NULL to skip      */
  int32_t               max_ctas;     /* 0: one CTA per SM; otherwise at most
                                         this many CTAs, leaving SMs free for
                                         work on other streams (e.g. an NCCL
                                         all-gather of a previous bucket)   */
  int32_t               reserved;
  int64_t*              step_counters; /* NULL: each descriptor's step is its
                                         row's `step`.  Non-NULL (capturable
                                         mode, for CUDA-graph replay): device
                                         step counts indexed by slot; a
                                         descriptor runs step t =
                                         step_counters[desc.slot] + 1 with row
                                         rows[desc.row + t - 1], and the call
                                         ends with that count = t.  A row
                                         index past n_rows skips the
                                         descriptor and raises
                                         LUMA_KERR_ROW_RANGE.  The reference
                                         keeps the same count in a device
                                         tensor (optimizer.py:382-387)       */
  const float*          grad_scale;   /* NULL, or a device float32 scalar c:
                                         every grad element g is used as
                                         round_to_grad_dtype(fl32(g) * c) —
                                         exactly torch._foreach_mul_(grads, c)
                                         as clip_grad_norm_ applies it
                                         (reference usage: bench_nanogpt.py:
                                         218, 225), fused into both passes
                                         instead of a separate pass over the
                                         grads; the grads are not modified  */
  float*                found_inf;    /* NULL, or a device float32 flag (the
                                         per-device found_inf tensor of
                                         torch.amp.GradScaler): pass 1 sets it
                                         to 1.0 if any grad element, as stored
                                         (before grad_scale), is inf or NaN,
                                         the check of
                                         torch._amp_foreach_non_finite_check_
                                         and_unscale_; if the flag is nonzero
                                         when pass 2 starts, the step changes
                                         no param, code or step count (the
                                         skipped optimizer.step() of
                                         GradScaler.step).  Reference usage:
                                         tests/test_mixed_precision.py:119-184,
                                         where GradScaler.unscale_ precedes
                                         opt.step() in a separate pass     */
} LumaStepArgs;

/*
 * Run one LUMA step for every descriptor: two launches on `stream`, no host
 * synchronisation, no allocation.  Descriptors whose row has step == 1 take
 * the reference's first-step path (zero-initialised moments, functional.py:
 * 183-228); the others decode their codes (functional.py:231-298).
 */
int luma_step(const LumaStepArgs* args, void* stream);

/*
 * luma_step_noalloc — the same step as luma_step for callers that cannot
 * allocate device memory of their own.  No counterpart in the reference.
 *
 * Who needs it: a host whose device memory is owned by another allocator
 * (a framework arena or caching allocator that has reserved the free HBM, an
 * FFI embedding with a fixed budget) or that must not call cudaMalloc from
 * its step thread (cudaMalloc/cudaFree synchronise the device).  Such a
 * caller still provides the tensors, the descriptor and row tables and the
 * LumaSlot state, but pass 1's per-tensor accumulators (the amax_m, amax_v
 * and done fields, which luma_step keeps in the caller's slots) come from a
 * scratch array built into the library: LUMA_NOALLOC_MAX_DESCS entries of
 * 16 bytes (64 KB), held by every GPU that loads the library until the
 * process exits.  The slots' accumulator fields are not touched.
 *
 * Limits and behaviour:
 *  - at most LUMA_NOALLOC_MAX_DESCS descriptors per call; larger tables are
 *    rejected with LUMA_ERR_INVALID (use luma_step);
 *  - the first call on a device looks up the scratch address on that device
 *    (cudaGetSymbolAddress with the device current); make that first call
 *    before any stream capture;
 *  - each call clears the scratch entries it uses (cudaMemsetAsync on
 *    `stream`), so a previous call's leftovers never leak into a new one;
 *  - all calls share the one array: calls whose kernels can overlap on the
 *    GPU (different streams without ordering) race and give wrong scales;
 *    serialise them;
 *  - nothing here allocates: no cudaMalloc, cudaFree or allocating library
 *    routine is called.
 */
#define LUMA_NOALLOC_MAX_DESCS 4096
int luma_step_noalloc(const LumaStepArgs* args, void* stream);

/*
 * Decode codes to float32 AdamW moments (reference optimizer.py:231-235 /
 * functional.py:113-126): exp_avg[i] = sign(q_m) expm1(|q_m| dm),
 * w = w_min exp(q_w dw), exp_avg_sq[i] = max(1/w - eps32, 0)^2, with the
 * float32 grid values dm = fl32(delta_m), w_min = fl32(w_min),
 * dw = fl32(delta_w) of _precompute(S_m, S_v, eps) and eps32 = fl32(eps).
 */
int luma_decode(const int16_t* q_m, const int16_t* q_w, int64_t numel,
                float dm, float w_min, float dw, float eps32,
                float* exp_avg, float* exp_avg_sq, void* stream);

/*
 * Quantize float32 AdamW moments into codes on `grid` (host pointer; built
 * for (S_m, S_v, eps) with S_m = max(max|m|, 1e-9), S_v = max(max v, 0)):
 * q_m from m, q_w from v (v >= 0), LogSR with the Philox stream keyed by
 * `seed` and counter offset `rng_offset` (even), or with the injected
 * uniforms u_m/u_w when both are non-NULL.  eps32 = fl32(eps), w_max =
 * fl32(1/eps).
 * Reference: optimizer.py:256-335 import_adamw_state, quantizer calls at
 * optimizer.py:315-321 (functional.py:133-176), seed (base_seed, step 0, idx).
 */
int luma_quantize(const float* m, const float* v, int64_t numel, const LumaGrid* grid,
                  float eps32, float w_max, int64_t seed, int64_t rng_offset,
                  const float* u_m, const float* u_w, int16_t* q_m, int16_t* q_w,
                  void* stream);

/*
 * Self-check of the library's branch-free correctly rounded reciprocal,
 * square root and quotient (used by the steady-state step loop) against CUDA's
 * IEEE intrinsics on the current GPU: n random operands of each over the
 * ranges where the step uses them.  Writes the mismatch counts (reciprocal,
 * square root, quotient) to mismatches[0..2] (host memory; all 0 on a correct
 * build) and synchronises `stream`.  No counterpart in the reference.
 */
int luma_arith_selfcheck(uint64_t n, uint64_t seed, uint64_t* mismatches, void* stream);

/*
 * Exhaustive check of the certified logarithms used by the steady-state step
 * loop: for every float a in [0, 2^-5] the momentum quantizer's series stays
 * within its stated bound of CUDA's log1pf(a), and for every float z in
 * [2^-1, 2^64] the preconditioner quantizer's approximation stays within its
 * bound of CUDA's logf(z).  Writes the violation counts to violations[0..1]
 * (all 0 on a correct build) and the largest errors seen to max_err[0..2]
 * (log1p relative; log absolute where |log| < 1; log relative elsewhere);
 * synchronises `stream`.  No counterpart in the reference.
 */
int luma_log_selfcheck(uint64_t* violations, double* max_err, void* stream);

/*
 * Peer memory for the copy-engine all-gather of the ZeRO-1 step (one process
 * per GPU).  A rank exports the device allocation holding its flat param
 * buffer (luma_ipc_export: IPC handle of the allocation and the byte offset of
 * `ptr` in it), the other ranks map it (luma_ipc_open / luma_ipc_close) and
 * push their updated pieces into it with luma_copy_async (one cudaMemcpyAsync:
 * the copy engines move the bytes, no SM is used).  The memory must come from
 * cudaMalloc (PyTorch's default caching allocator does).  No counterpart in the
 * reference, whose optimizer never exchanges data (optimizer.py:399-407).
 */
typedef struct LumaIpcHandle {
  unsigned char bytes[64];
} LumaIpcHandle;

int luma_ipc_export(const void* ptr, LumaIpcHandle* handle, uint64_t* offset);
int luma_ipc_open(const LumaIpcHandle* handle, void** base);
int luma_ipc_close(void* base);
int luma_copy_async(void* dst, const void* src, uint64_t bytes, void* stream);

/*
 * Launch shape of the step kernels, for tuning reports (reference
 * config.py:35-73 get_kernel_config): writes out[0..7] = pass-1 threads per
 * CTA, pass-1 elements per thread per iteration, pass-1 staging stages,
 * pass-2 threads per CTA, pass-2 elements per thread per iteration, pass-2
 * staging stages, CTAs per SM, minimum segment length (elements) for the
 * shared-memory decode table; returns the number written (<= n).
 */
int luma_launch_config(int32_t* out, int n);

/*
 * NVLink multicast copy: `bytes` bytes from `src` (this GPU's memory) to
 * `mc_dst`, an address in a multicast (NVLS) mapping, with multimem stores
 * on `stream` — every GPU bound to the multicast object receives the bytes at
 * the same offset, the NVSwitch doing the fan-out (the all-gather of a ZeRO
 * piece as one write).  Both addresses and `bytes` must be multiples of 16.
 * Ends with a system-scope fence; the caller orders the peers' reads after it
 * (a barrier).  No counterpart in the reference (optimizer.py:399-407 leaves
 * gathers to FSDP).
 */
int luma_mc_copy(void* mc_dst, const void* src, uint64_t bytes, void* stream);

/* ABI version (LUMA_ABI_VERSION). */
int luma_abi_version(void);

/*
 * Layout check for FFI callers: writes sizeof of LumaTensorDesc, LumaStepRow,
 * LumaGrid, LumaSlot, LumaStepArgs into out[0..4] and returns 5 (or fewer if
 * n < 5).
 */
int luma_struct_sizes(int64_t* out, int n);

/* Message of the last failed call on this thread ("" if none). */
const char* luma_last_error(void);

/*
 * Kernel error flags of the current device (bits below), raised by the step
 * kernels for conditions only the device sees: in capturable mode, a step
 * count whose row lies past the row table (the descriptor was skipped).
 * Synchronises the device; with `clear` != 0 the flags are reset afterwards.
 */
#define LUMA_KERR_ROW_RANGE 1u
int luma_error_flags(uint32_t* out, int clear);

#ifdef __cplusplus
}
#endif

#endif /* LUMA_B200_H */
