/*
 * hxm.h — C ABI of the B200 (sm_100a) recurrent hot path of the hybrid
 * Mamba / xLSTM model (selective scan, chunkwise mLSTM, Mamba-2 SSD chunked
 * scan, sLSTM recurrence).
 *
 * Conventions shared by every entry point
 *   - All tensors are caller-owned DEVICE buffers passed as raw pointers plus
 *     strides counted in ELEMENTS (not bytes).  Nothing on the hot path
 *     allocates; an entry point that needs scratch says so through its
 *     *_workspace_size() companion and takes a caller-owned workspace.
 *   - `stream` is a cudaStream_t passed as void* (0 = legacy default stream).
 *     Work is enqueued asynchronously; no entry point synchronizes the host.
 *   - Entry points never throw and never abort: they return an hxm_status.
 *     On failure hxm_last_error_string() returns a thread-local message.
 *   - Argument structs start with `struct_size` = sizeof(the struct) so the
 *     ABI can grow; a caller built against an older header is rejected with
 *     HXM_EBADARG instead of being misread.
 *   - Stateless and re-entrant; one process per GPU; the device is the
 *     caller's current device.
 */
#ifndef HXM_H_
#define HXM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HXM_ABI_VERSION 1

typedef enum hxm_status {
  HXM_OK = 0,
  HXM_EBADARG = 1,      /* shape / stride / dtype / pointer validation failed   */
  HXM_EUNSUPPORTED = 2, /* valid request this build has no kernel for           */
  HXM_ECUDA = 3,        /* a CUDA runtime call or kernel launch failed          */
  HXM_ETIMEOUT = 4      /* a bounded device-side wait gave up (error flag set)  */
} hxm_status;

typedef enum hxm_dtype { HXM_F32 = 0, HXM_BF16 = 1, HXM_F16 = 2 } hxm_dtype;

/* ------------------------------------------------------------------------ */
/* Library                                                                   */
/* ------------------------------------------------------------------------ */

/* ABI version compiled into the library (HXM_ABI_VERSION). */
int hxm_abi_version(void);

/* Thread-local description of the last failure in this thread ("" if none). */
const char* hxm_last_error_string(void);

/* ------------------------------------------------------------------------ */
/* 1. Selective scan (Mamba S6)                                               */
/*                                                                           */
/* Replaces selective_scan / SelectiveScanFunction.forward                   */
/*   (hybrid_xmamba/kernels/selective_scan/scan_interface.py:17-60,155-180)  */
/* and its CPU loop selective_scan_pytorch (scan_interface.py:103-152), plus */
/* the CUDA kernel selective_scan_triton (scan_triton.py:408-500).           */
/*                                                                           */
/* Per (b, d) channel, state h[n] (fp32, starts at h0 or 0):                  */
/*   delta   = softplus(dt + delta_bias)   (softplus/bias optional)          */
/*   euler:  h = exp(delta*A[d,n]) * h + delta * B[b,t,n] * u              */
/*   zoh:    h = exp(dA) * h + Bbar * u, Bbar = (exp(dA)-1)/A * B, or         */
/*           delta*B when |delta*A| < 0.01 (scan_triton.py:135-160)           */
/*   y       = sum_n C[b,t,n] h[n] + D[d] * u                                */
/*   z_mode: 0 none, 1 y*z (scan_interface.py:57-58), 2 y*silu(z)            */
/* Logical shapes: u, delta, z, y (batch, seqlen, dim); A (dim, dstate);     */
/* B, C (batch, seqlen, dstate); D, delta_bias (dim); h0, hT                 */
/* (batch, dim, dstate) fp32 contiguous.  Any element strides are accepted;  */
/* the fast path wants either the time axis or the channel axis unit-stride. */
/* ------------------------------------------------------------------------ */
typedef struct hxm_scan_args {
  size_t struct_size;
  int32_t batch, seqlen, dim, dstate;
  hxm_dtype io_dtype;       /* dtype of u, delta, z, B, C, y                 */
  const void* u;      int64_t u_stride[3];      /* (b, t, d)                 */
  const void* delta;  int64_t delta_stride[3];  /* (b, t, d)                 */
  const float* A;     int64_t A_stride[2];      /* (d, n)   fp32             */
  const void* B;      int64_t B_stride[3];      /* (b, t, n)                 */
  const void* C;      int64_t C_stride[3];      /* (b, t, n)                 */
  const float* D;                               /* (d) fp32 or NULL          */
  const void* z;      int64_t z_stride[3];      /* (b, t, d) or NULL         */
  const float* delta_bias;                      /* (d) fp32 or NULL          */
  void* y;            int64_t y_stride[3];      /* (b, t, d)                 */
  const float* h0;                              /* (b, d, n) fp32 or NULL    */
  float* hT;                                    /* (b, d, n) fp32 or NULL    */
  int32_t z_mode;           /* 0 none, 1 multiply, 2 silu-gate               */
  int32_t delta_softplus;   /* 0/1                                           */
  int32_t discretization;   /* 0 euler (reference CPU path), 1 zoh           */
  void* workspace;          /* hxm_selective_scan_workspace_size() bytes, or */
  size_t workspace_bytes;   /* NULL / 0: one pass (no time segments)         */
} hxm_scan_args;

hxm_status hxm_selective_scan_fwd(const hxm_scan_args* args, void* stream);
/* Scratch the forward can use for time segments (0 = none): when the grid   */
/* would not fill the GPU (few batch rows x channels, e.g. one shard of a   */
/* batch split over GPUs), bf16 Euler requests run the sequence as up to 16 */
/* parallel segments after a state-only pass; with workspace == NULL or too */
/* small the forward runs one pass.  17 floats per (batch, channel) and     */
/* segment boundary.                                                         */
size_t hxm_selective_scan_workspace_size(const hxm_scan_args* args);

/* Selective scan backward (Euler discretization).                           */
/* Replaces the recompute-under-autograd backward of SelectiveScanFunction   */
/*   (hybrid_xmamba/kernels/selective_scan/scan_interface.py:62-100).        */
/* Inputs as hxm_scan_args (u, delta, A, B, C, D, z, delta_bias, h0, z_mode, */
/* delta_softplus; discretization must be 0) plus dout (b, t, d) strided.    */
/* Outputs, fp32 and dense: du, ddelta (delta's pre-softplus input), dz      */
/* (b, t, d); dA (d, n); dB, dC (b, t, n); dD, ddelta_bias (d); dh0 (b, d, n).*/
/* Any output may be NULL when not needed (the sums are still consistent).   */
/* The per-channel states are recomputed from checkpoints every 16 steps     */
/* kept in a workspace of hxm_selective_scan_bwd_workspace_size() bytes.     */
typedef struct hxm_scan_bwd_args {
  hxm_scan_args fwd;        /* fwd.struct_size = sizeof(hxm_scan_args); y, hT unused */
  size_t struct_size;       /* sizeof(hxm_scan_bwd_args)                     */
  const void* dout;   int64_t dout_stride[3];
  float* du; float* ddelta; float* dz;
  float* dA; float* dB; float* dC; float* dD; float* ddelta_bias; float* dh0;
  void* workspace; size_t workspace_bytes;
} hxm_scan_bwd_args;

size_t hxm_selective_scan_bwd_workspace_size(const hxm_scan_bwd_args* args);
hxm_status hxm_selective_scan_bwd(const hxm_scan_bwd_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* 2. mLSTM chunkwise forward ("TFLA")                                        */
/*                                                                           */
/* Replaces apply_tfla / TFLAFunction.forward / tfla_forward_pytorch         */
/*   (hybrid_xmamba/kernels/tfla/tfla_interface.py:18-49,84-139,142-163)     */
/* and the intended chunkwise kernels of tfla_triton.py:23-359.              */
/*                                                                           */
/* Per (b, h): C (dqk x dv), n (dqk) with                                     */
/*   C_t = f_t * C_{t-1} + i_t * k_t v_t^T,  n_t = f_t * n_{t-1} + i_t * k_t */
/*   h_t = (q_t^T C_t) / max(q_t . n_t, 1)                                   */
/* Gates are given as PRE-activations in log space:                          */
/*   log_i = input-gate preactivation (i = exp(log_i)),                      */
/*   log_f = log forget gate (f = exp(log_f), e.g. logsigmoid(preact)).      */
/* gate_mode 0: per-head scalar gates (b, h, t); 1: per-channel gates        */
/* (b, h, t, dqk) as in mLSTMBlock (mlstm_block.py:117-129).                 */
/* The state is kept stabilized: C = exp(m) * Cs, n = exp(m) * ns.  Inputs    */
/* C0/n0/m0 and outputs CT/nT/mT use that representation (NULL = zero).      */
/* q, k, v, h: (b, h, t, d) with arbitrary (b, h) strides, unit d stride and */
/* a time stride (*_tstride; 0 = d, one dense (t, d) panel per head), so     */
/* (b, t, h, d) projection outputs are passed without a transpose.           */
/* Requires a workspace of hxm_mlstm_workspace_size() bytes.                 */
/* Any gate values: (b, h) pairs whose chunk scaling would leave the fp32    */
/* range on the key-streaming path (e.g. a 128-step chunk whose forget gates */
/* sum below about -128, or f = 0) are detected on the device and run by the */
/* exact recurrent kernel within the same call (no host synchronization).   */
/* ------------------------------------------------------------------------ */
typedef struct hxm_mlstm_args {
  size_t struct_size;
  int32_t batch, heads, seqlen, dqk, dv;
  int32_t chunk;            /* 0 or 128: the kernels' time chunk (the result */
                            /* does not depend on it); others: EUNSUPPORTED  */
  int32_t gate_mode;        /* 0 scalar per head, 1 per channel              */
  hxm_dtype io_dtype;       /* q, k, v, h                                    */
  const void* q; int64_t q_stride[2];   /* (b, h) strides; time: q_tstride   */
  const void* k; int64_t k_stride[2];
  const void* v; int64_t v_stride[2];
  const float* log_i;  int64_t i_stride[2];   /* (b, h); time: i_tstride; d dense */
  const float* log_f;  int64_t f_stride[2];
  void* h;   int64_t h_stride[2];
  const float* C0; const float* n0; const float* m0;  /* (b,h,dqk,dv) (b,h,dqk) (b,h) fp32 or NULL */
  float* CT; float* nT; float* mT;                    /* same shapes, or NULL */
  void* workspace; size_t workspace_bytes;
  /* time strides in elements; 0 = dense (dqk for q, k; dv for v, h; 1 per-head */
  /* or dqk per-channel gates)                                                 */
  int64_t q_tstride, k_tstride, v_tstride, h_tstride, i_tstride, f_tstride;
  /* Bounded device waits of the tensor-core kernels: error_flag (device int */
  /* or NULL) is set to 1 when one gives up (its outputs are then not       */
  /* written); wait_limit_cycles bounds each wait in SM clock cycles        */
  /* (0 = 4e9, about 2 s; < 0: every wait gives up at once, which exercises */
  /* the error path — the kernel still drains its own MMAs and loads).      */
  int32_t* error_flag;
  int64_t wait_limit_cycles;
} hxm_mlstm_args;

size_t hxm_mlstm_workspace_size(const hxm_mlstm_args* args);
hxm_status hxm_mlstm_chunkwise_fwd(const hxm_mlstm_args* args, void* stream);

/* No counterpart in the reference.  Same computation as
 * hxm_mlstm_chunkwise_fwd on its key-streaming tensor-core path (bf16,
 * dqk 128/256/512, per-head or per-channel gates), for callers that cannot
 * allocate device memory at call time (plugin hosts whose execute callbacks
 * forbid cudaMalloc, programs that pre-reserve all device memory): it needs
 * no workspace — args->workspace is ignored — and allocates nothing.  Its
 * scratch is one library-owned 32 MiB device array per GPU, held until exit;
 * requests needing more return HXM_EBADARG.  The first call on a device looks
 * up the array's address and keeps it for the life of the process (make it
 * before any stream capture; a cudaDeviceReset afterwards is not supported);
 * calls that overlap on the GPU race on the shared array. */
hxm_status hxm_mlstm_chunkwise_fwd_noalloc(const hxm_mlstm_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* 2b. mLSTM chunkwise backward (zero initial state)                          */
/*                                                                           */
/* Replaces the recompute-under-autograd backward of TFLAFunction            */
/*   (hybrid_xmamba/kernels/tfla/tfla_interface.py:52-81), which re-runs the */
/* step loop tfla_forward_pytorch (:84-139) under autograd.                  */
/* Chunkwise form, per (b, h), chunk of `chunk` steps and key channel j, with*/
/* b_t = sum of log_f over the chunk's steps up to t, g = b at the chunk's   */
/* last step and rho = g / 2:                                                */
/*   Qs_t = q_t e^(b_t - rho),  Ks_t = k_t e^(log_i_t + rho - b_t)            */
/* (intra-chunk weights Qs_t . Ks_s; the state entering the next chunk is    */
/* e^g C + e^rho Ks^T [v | 1], n riding as the column of ones).  The batched */
/* chunk GEMMs between the calls below are the caller's (hxm_chunk_gemm).    */
/*   hxm_mlstm_bwd_prepare: q, k (b, h, t) strided with dense dqk, log gates */
/*     (b, h, t) strided, per head (gate_mode 0) or per channel (1, dense    */
/*     dqk) -> q_scaled, k_scaled (b, h, nchunks*chunk, dqk), zero past      */
/*     seqlen; rho, e_rho = e^rho, e_g = e^g (b, h, nchunks, dqk).  fp32,     */
/*     dense.                                                                */
/*   hxm_mlstm_bwd_finalize: dq_scaled = dL/dQs, dk_scaled = dL/dKs (layout   */
/*     of q_scaled) plus q_scaled, k_scaled, rho and the gates ->             */
/*     dq = e^(b - rho) dL/dQs, dk = e^(log_i + rho - b) dL/dKs,              */
/*     dlog_i = Ks . dL/dKs (per channel), and                               */
/*     dlog_f_t = chunk_dg + sum over s >= t in the chunk of                 */
/*                (Qs . dL/dQs - Ks . dL/dKs)_s,                             */
/*     d_i = k e^(rho - b) dL/dKs (the gradient for the gate value i, with no */
/*     division by i), all (b, h, seqlen, dqk) fp32 dense.  chunk_dg          */
/*     (b, h, nchunks, dqk), an input: the gradient for the chunk's total     */
/*     log forget gate through the state it passes on, i.e. per key row the   */
/*     inner product of the state leaving the chunk with its adjoint (zero    */
/*     for the last chunk).  Per-head gate gradients are the sums over dqk.   */
typedef struct hxm_mlstm_bwd_args {
  size_t struct_size;
  int32_t batch, heads, seqlen, dqk, chunk;
  int32_t gate_mode;        /* 0 per head, 1 per channel                     */
  hxm_dtype io_dtype;       /* q, k                                          */
  const void* q; int64_t q_stride[3];          /* (b, h, t) element strides  */
  const void* k; int64_t k_stride[3];
  const float* log_i; int64_t i_stride[3];     /* (b, h, t)                  */
  const float* log_f; int64_t f_stride[3];
  float* q_scaled; float* k_scaled;
  float* rho; float* e_rho; float* e_g;
  float* q_decayed; float* k_decayed;  /* prepare, optional (NULL = skip):    */
                            /* q e^b and k e^(log_i + g - b), layout of q_scaled */
  void* split_planes;       /* optional bf16 (8, b, h, nchunks*chunk, dqk):   */
                            /* high / low parts (x = hi + lo to ~2^-16) of    */
                            /* q_scaled, k_scaled, q_decayed, k_decayed in    */
                            /* that order, the tensor-core chunk GEMMs'       */
                            /* operands.  prepare writes them (q_scaled ...   */
                            /* may then be NULL); finalize reads q_scaled,    */
                            /* k_scaled from them when those are NULL.        */
  const float* dq_scaled; const float* dk_scaled;
  const float* chunk_dg;
  float* dq; float* dk; float* dlog_i; float* dlog_f;
  float* d_i;               /* (b, h, seqlen, dqk) or NULL: dL/di, i = e^log_i */
} hxm_mlstm_bwd_args;

hxm_status hxm_mlstm_bwd_prepare(const hxm_mlstm_bwd_args* args, void* stream);
hxm_status hxm_mlstm_bwd_finalize(const hxm_mlstm_bwd_args* args, void* stream);

/* Output-side gradients of the chunkwise backward, one row per step t of    */
/* each (b, h), t < padded_len (seqlen rounded up to whole chunks):          */
/*   normalize: dnum = dh / max(den, 1), dden = -[den >= 1] dnum . num /     */
/*              max(den, 1), from outputs[row] = [num (dv) | den | ...];     */
/*   else:      dnum = dh, dden = 0;                                         */
/* written as out[row] = [dnum | dden | 0 ...] (width floats; zero rows past */
/* seqlen).  outputs, out: (b, h, padded_len, width) fp32 dense; dh          */
/* (b, h, t) element strides, dense dv, io dtype.  Replaces the clamp branch */
/* of the reference's recompute-under-autograd backward (tfla_interface.py: */
/* 52-81 differentiating :133-137).  out_hi / out_lo (optional, bf16,       */
/* layout of out): the same rows as a split operand (hi + lo to ~2^-16);     */
/* out may then be NULL.                                                     */
typedef struct hxm_mlstm_bwd_norm_args {
  size_t struct_size;
  int32_t batch, heads, seqlen, padded_len, dv, width;
  int32_t normalize;
  hxm_dtype io_dtype;       /* dh                                            */
  const float* outputs;
  const void* dh; int64_t dh_stride[3];
  float* out;
  void* out_hi; void* out_lo;
} hxm_mlstm_bwd_norm_args;

hxm_status hxm_mlstm_bwd_normalizer(const hxm_mlstm_bwd_norm_args* args, void* stream);

/* Exclusive chunk-level recurrence, in place, for the chunkwise backward:   */
/* per group and element (r, c), s = 0 and for each chunk k in order         */
/* (reverse = 0) or in reverse (reverse = 1):                                 */
/*   y = x[k, r, c];  x[k, r, c] = s;  s = decay[k, r] * s + y               */
/* so x becomes the states entering each chunk (forward) or the adjoints     */
/* leaving each chunk (reverse); with `scaled`, also the row-scaled copy     */
/* scaled[k, r, c] = scale[k, r] * x[k, r, c] of the output.                 */
/* x (groups, nchunks, rows, cols), decay                                    */
/* (groups, nchunks, rows) or NULL (= 1), fp32 dense.  No reference          */
/* counterpart: the reference's backward has no chunk states.                */
typedef struct hxm_chunk_scan_args {
  size_t struct_size;
  int64_t groups;
  int32_t nchunks, rows, cols;
  float* x;
  const float* decay;
  int32_t reverse;
  const float* scale;       /* (groups, nchunks, rows) or NULL              */
  float* scaled;            /* layout of x, or NULL: scale[k, r] * x_out[k] */
  void* scaled_hi;          /* optional bf16, layout of x: the scaled copy  */
  void* scaled_lo;          /* (x_out when scale is NULL) as high / low     */
                            /* parts, a split operand (hi + lo to ~2^-16)   */
  /* Row mode (scaled_hi set, rows x cols with cols % 4 == 0 and cols <= 640): */
  /* with skip_state = 1, x is only read (the exclusive states go to the       */
  /* split copy alone); with dot_out, also                                     */
  /*   dot_out[g, k, r] = sum_c x_out[g, k, r, c] * (dot_hi + dot_lo)[g, k + 1, r, c] */
  /*                      / dot_scale[g, k + 1, r]   (dot_scale NULL = 1)      */
  /* and 0 for the last chunk: the chunk gradient of hxm_chunk_state_dot from  */
  /* the adjoint scan and the split copy the state scan wrote.                 */
  int32_t skip_state;
  const void* dot_hi; const void* dot_lo;
  const float* dot_scale;
  float* dot_out;           /* (groups, nchunks, rows)                        */
} hxm_chunk_scan_args;

hxm_status hxm_chunk_state_scan(const hxm_chunk_scan_args* args, void* stream);

/* Per chunk and row, the inner product of the adjoint leaving the chunk     */
/* with the state leaving it (the state entering the next chunk):            */
/*   out[g, k, r] = sum_c adj[g, k, r, c] * state[g, k + 1, r, c],           */
/* 0 for the last chunk: the gradient for the chunk's total log forget gate  */
/* (chunk_dg of hxm_mlstm_bwd_finalize).  adj, state (groups, nchunks, rows, */
/* cols), out (groups, nchunks, rows), fp32 dense.  No reference counterpart.*/
typedef struct hxm_chunk_dot_args {
  size_t struct_size;
  int64_t groups;
  int32_t nchunks, rows, cols;
  const float* adj;
  const float* state;
  float* out;
} hxm_chunk_dot_args;

hxm_status hxm_chunk_state_dot(const hxm_chunk_dot_args* args, void* stream);

/* Gate-scaled split operands of the chunkwise backward passes: for batch b,*/
/* step t < padded_len and column c,                                          */
/*   v = x[b, t, c] * scale[b, t, c / group]   (t < seqlen; scale NULL = 1)  */
/*   v = 0                                      (seqlen <= t < padded_len)    */
/*   hi[b, t, c] = bf16(v),  lo[b, t, c] = bf16(v - hi)  (lo may be NULL)     */
/* x: io dtype, element strides (b, t), unit column stride; scale fp32 dense */
/* (batch, padded_len, cols / group); hi, lo bf16 dense (batch, padded_len,  */
/* cols).  One pass in place of the gate products, padding copies and the   */
/* high / low rounding of the chunk GEMMs' operands (e.g. alpha x and beta dy */
/* of the SSD backward, i k and e^b q of the per-head mLSTM backward).        */
typedef struct hxm_scale_split_args {
  size_t struct_size;
  int32_t batch, seqlen, padded_len, cols, group;
  hxm_dtype io_dtype;
  const void* x; int64_t x_stride[2];
  const float* scale;
  void* hi; void* lo;
} hxm_scale_split_args;

hxm_status hxm_scale_split(const hxm_scale_split_args* args, void* stream);

/* Batched chunk GEMM on the tensor cores (tcgen05; bf16 operands, fp32      */
/* accumulation) for the chunk contractions of the chunkwise backward passes */
/* (the intra-chunk products of the reference's recompute-under-autograd    */
/* backward, tfla_interface.py:52-81 differentiating :113-137).  Per group g:*/
/*   D = alpha * sum_{p < nprod} op(A_p) op(B_p)    (m x n, nprod 1 to 4)     */
/* then: mask = 1 zeroes D[r, c] for c > r (a chunk's causal step matrix);   */
/* with `decay`, D[r, c] *= exp(decay[g, r] - decay[g, c]) for c <= r;       */
/* accumulate = 1 adds the fp32 output's current value; D is stored to `out` */
/* (fp32) and / or `out_bf16` (with out_bf16_lo, also the low part: high +  */
/* low carry ~16 mantissa bits, a split operand for the next products).  Each operand is a stored bf16 matrix per     */
/* group (rows x cols, unit column stride, 16-byte aligned base, row and     */
/* group strides multiples of 8 elements); trans = 1 uses it transposed, so  */
/* op(A) is m x K and op(B) K x n.  groups <= 2^24.  Outputs: unit column   */
/* stride, fp32 16-byte aligned / bf16 8-byte aligned, row and group strides */
/* multiples of 4 elements.                                                  */
typedef struct hxm_gemm_operand {
  const void* ptr;
  int64_t group_stride, row_stride;   /* elements                            */
  int32_t rows, cols;                 /* stored extent per group             */
  int32_t trans;
} hxm_gemm_operand;

typedef struct hxm_chunk_gemm_args {
  size_t struct_size;
  int64_t groups;
  int32_t m, n, nprod;
  hxm_gemm_operand a[4], b[4];
  float alpha;
  int32_t mask;
  const float* decay; int64_t decay_stride;   /* (groups, m) per step, or NULL */
  int32_t accumulate;
  float* out;     int64_t out_group_stride, out_row_stride;
  void* out_bf16; int64_t outb_group_stride, outb_row_stride;
  void* out_bf16_lo;          /* or NULL: bf16(D - bf16(D)), strides of out_bf16 */
  int32_t* error_flag;        /* set to 1 when a bounded wait gave up, or NULL */
  int64_t wait_limit_cycles;  /* 0: default (~2 s)                           */
} hxm_chunk_gemm_args;

hxm_status hxm_chunk_gemm(const hxm_chunk_gemm_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* 3. Mamba-2 SSD chunked scan (ngroups = 1)                                  */
/*                                                                           */
/* No function of the reference computes this; its arithmetic is the Euler   */
/* selective scan (scan_interface.py:103-152) with channel d = (head, p),    */
/* A[d, :] = A[head], delta[b, t, d] = dt[b, t, head] and B, C shared.       */
/*   h[p, n] = exp(dt*A) h[p, n] + dt * x[p] * B[n];  y[p] = C.h[p,:] + D*x  */
/* x, y (b, t, heads, p) bf16; B, C (b, t, n) bf16; dt (b, t, heads) fp32;   */
/* A, D, dt_bias (heads) fp32; state (b, heads, p, n) fp32.  All dense.      */
/* ------------------------------------------------------------------------ */
typedef struct hxm_ssd_args {
  size_t struct_size;
  int32_t batch, seqlen, heads, headdim, dstate;
  int32_t chunk;            /* 0 or 128: the kernel's time chunk (the result */
                            /* does not depend on it); others: EUNSUPPORTED  */
  hxm_dtype io_dtype;       /* x, B, C, y                                    */
  const void* x; const float* dt; const float* A;
  const void* B; const void* C;
  const float* D;           /* (heads) or NULL                               */
  const float* dt_bias;     /* (heads) or NULL                               */
  int32_t dt_softplus;
  void* y;
  const float* h0;          /* (b, heads, p, n) or NULL                      */
  float* hT;                /* (b, heads, p, n) or NULL                      */
  void* workspace; size_t workspace_bytes;
  int32_t* error_flag;      /* device int set to 1 if a bounded wait gave up */
  int64_t wait_limit_cycles;/* per wait, SM clock cycles (0 = 4e9, ~2 s;     */
                            /* < 0: every wait gives up at once)             */
} hxm_ssd_args;

size_t hxm_ssd_workspace_size(const hxm_ssd_args* args);

/* SSD backward, per-head intra-chunk terms (no reference counterpart: the    */
/* reference has no SSD; its arithmetic is the Euler scan of                 */
/* scan_interface.py:132-150 with channel (head, p)).  Per (batch, chunk) of */
/* `chunk` (32 or 64) steps and head h, with bcum the in-chunk prefix sum of */
/* the head's log decay dt*A, cb = C B^T of the chunk and G = dL/dS_h:       */
/*   S[h, t, s]  = cb[t, s] e^(bcum_t - bcum_s) dt_s   (s <= t, else 0)       */
/*   M[t, s]     = sum_h G[h, t, s] e^(bcum_t - bcum_s) dt_s                  */
/*   ddt[h, s]   = sum_t G[h, t, s] cb[t, s] e^(bcum_t - bcum_s)              */
/*   db[h, t]    = rowsum(W)[t] - colsum(W)[t], W = G * S without its diagonal*/
/* cb, M (batch*nchunks, chunk, chunk); bcum, dt (batch*nchunks, chunk,      */
/* heads); dS = G and S (batch*nchunks, heads, chunk, chunk); ddt, db        */
/* (batch*nchunks, heads, chunk).  fp32, dense.                               */
typedef struct hxm_ssd_bwd_intra_args {
  size_t struct_size;
  int32_t batch, nchunks, heads, chunk;
  const float* cb; const float* bcum; const float* dt; const float* dS;
  float* S; float* M; float* ddt; float* db;
} hxm_ssd_bwd_intra_args;

hxm_status hxm_ssd_bwd_intra(const hxm_ssd_bwd_intra_args* args, void* stream);

/* SSD backward, per (batch, chunk, step t, head h) row of headdim values    */
/* (no reference counterpart, as above):                                     */
/*   dx[b, t_global, h, :] = dxi + alpha[t, h] * BY + D[h] * dy               */
/*   xby = x . BY,  dycz = dy . CZ,  dyx = dy . x        (per row)            */
/* xh, dyh, dxi (batch*nchunks, heads, chunk, headdim) head-major; BY, CZ    */
/* (batch*nchunks, chunk, heads, headdim); alpha, xby, dycz, dyx             */
/* (batch*nchunks, chunk, heads); D (heads) or NULL; dyx may be NULL;        */
/* dx (batch, seqlen, heads, headdim), rows past seqlen not written.  fp32.  */
typedef struct hxm_ssd_bwd_rows_args {
  size_t struct_size;
  int32_t batch, nchunks, chunk, heads, headdim, seqlen;
  const float* xh; const float* dyh; const float* dxi;
  const float* BY; const float* CZ; const float* alpha; const float* D;
  float* dx; float* xby; float* dycz; float* dyx;
} hxm_ssd_bwd_rows_args;

hxm_status hxm_ssd_bwd_rows(const hxm_ssd_bwd_rows_args* args, void* stream);
hxm_status hxm_ssd_chunk_scan_fwd(const hxm_ssd_args* args, void* stream);

/* ------------------------------------------------------------------------ */
/* 4. sLSTM recurrence                                                        */
/*                                                                           */
/* Replaces the inline loop of sLSTMBlock.forward                            */
/*   (hybrid_xmamba/layers/slstm_block.py:91-127) including its fused        */
/* RMSNorm over head_dim (layers/normalization.py:32-34).                    */
/* Per (b, head) with hd = head_dim and gate pre-activations                 */
/*   g_t = gates_pre[b, t, head, :, :] + R[head]^T h_{t-1}    (4 x hd)       */
/* ordered [i | f | o | ctilde] as gates.chunk(4, -1) splits them:           */
/*   i = exp(g_i) (or sigmoid), f = sigmoid(g_f), o = sigmoid(g_o),          */
/*   c = f*c + i*tanh(g_c);  h = o * tanh(w * c / sqrt(mean(c^2) + eps))     */
/* R (heads, hd, 4*hd) bf16 or NULL (the reference has no recurrent R).      */
/* gates_pre (b, t, heads, 4, hd) bf16/fp32 dense; h_out (b, t, heads, hd);  */
/* h0, c0, hT, cT (b, heads, hd) fp32 or NULL: the true hidden and cell      */
/* states, i.e. the reference's cache['h'], cache['c'] (slstm_block.py:      */
/* 105-107,139-141).  Exponential input gates are stabilized internally per  */
/* channel; head_dim 128 / 256 with R run the 8-CTA cluster kernel.          */
/* error_flag: device int set to 1 if a bounded cross-CTA wait gave up.      */
typedef struct hxm_slstm_args {
  size_t struct_size;
  int32_t batch, seqlen, heads, head_dim;
  hxm_dtype io_dtype;       /* gates_pre, h_out                              */
  const void* gates_pre;
  const void* R;            /* bf16 (heads, hd, 4*hd) or NULL                */
  const float* norm_weight; /* (hd)                                          */
  float eps;
  int32_t exponential_gate; /* 1: i = exp, 0: i = sigmoid                    */
  void* h_out;
  const float* h0; const float* c0;
  float* hT; float* cT;
  int32_t* error_flag;      /* device int or NULL                            */
  int64_t wait_limit_cycles;/* per cross-CTA wait, SM cycles (0 = 4e9, ~2 s; */
                            /* < 0: the first exchange is waited for -limit */
                            /* cycles before any CTA sends, so it runs out)  */
} hxm_slstm_args;

hxm_status hxm_slstm_scan_fwd(const hxm_slstm_args* args, void* stream);

/* ---- causal depthwise conv1d (+ SiLU) ------------------------------------ */
/* Replaces the Mamba pre-scan convolution of MambaBlock.forward             */
/*   (hybrid_xmamba/layers/mamba_block.py:101-104): nn.Conv1d(groups=dim,    */
/*   padding=width-1) trimmed to the first seqlen outputs, then SiLU:        */
/*   out[b, t, c] = act(bias[c] + sum_k weight[c, k] * x[b, t - width+1+k, c]) */
/* with x[b, t < 0, c] taken from init_state (or zero).                      */
/* x, out: (batch, seqlen, channels) element strides, bf16 / fp32; the       */
/* channel stride should be 1 (other strides run a slower element kernel).   */
/* weight (channels, width) fp32 dense; bias (channels) fp32 or NULL;        */
/* width 1..4.  init_state / final_state: (batch, channels, width-1) in the  */
/* io dtype, dense, or NULL: the width-1 inputs before t = 0 / the last      */
/* width-1 inputs (for continuing a sequence).                               */
typedef struct hxm_conv1d_args {
  size_t struct_size;
  int32_t batch, seqlen, channels, width;
  hxm_dtype io_dtype;
  const void* x;       int64_t x_stride[3];
  const float* weight;
  const float* bias;
  void* out;           int64_t out_stride[3];
  const void* init_state;
  void* final_state;
  int32_t activation;  /* 0 none, 1 SiLU                                     */
} hxm_conv1d_args;

hxm_status hxm_causal_conv1d_fwd(const hxm_conv1d_args* args, void* stream);

/* ---- RMSNorm (optionally fused with the residual add before it) ---------- */
/* Replaces RMSNorm.forward (hybrid_xmamba/layers/normalization.py:32-34):   */
/*   out = weight * s / sqrt(mean(s^2) + eps)   over the last dim            */
/* where s = x, or s = x + residual (the residual adds of HybridBlock.forward,*/
/* hybrid_xmamba/layers/hybrid_block.py:125,132) rounded to the io dtype and  */
/* also written to sum_out when it is not NULL (it may alias x or residual). */
/* Rows of dim contiguous elements, bf16 / fp32, row strides in elements;    */
/* weight (dim) fp32 or NULL (ones).                                         */
typedef struct hxm_rmsnorm_args {
  size_t struct_size;
  int64_t rows;
  int32_t dim;
  hxm_dtype io_dtype;
  const void* x;        int64_t x_row_stride;
  const void* residual; int64_t residual_row_stride;
  void* sum_out;        int64_t sum_row_stride;
  const float* weight;
  float eps;
  void* out;            int64_t out_row_stride;
} hxm_rmsnorm_args;

hxm_status hxm_rmsnorm_fwd(const hxm_rmsnorm_args* args, void* stream);

/* ---- mLSTM gate prologue / epilogue ---------------------------------------- */
/* Replace the element-wise gate work of mLSTMBlock.forward                  */
/* (hybrid_xmamba/layers/mlstm_block.py:117-119,138-141) around the           */
/* recurrence, one HBM pass each, on (rows, dim) matrices with row strides   */
/* in elements and unit column stride:                                       */
/*   prologue: log_i = i_pre (fp32), log_f = logsigmoid(f_pre) (fp32)        */
/*             (the log-space gates of hxm_mlstm_chunkwise_fwd);             */
/*   epilogue: out = h * sigmoid(o_pre) * sigmoid(x_gate).                    */
/* i_pre, f_pre, o_pre, x_gate, h, out: io dtype (bf16 / fp32).              */
typedef struct hxm_mlstm_gates_args {
  size_t struct_size;
  int64_t rows;
  int32_t dim;
  hxm_dtype io_dtype;
  /* prologue */
  const void* i_pre; int64_t i_row_stride;
  const void* f_pre; int64_t f_row_stride;
  float* log_i;      int64_t log_i_row_stride;
  float* log_f;      int64_t log_f_row_stride;
  /* epilogue */
  const void* h;      int64_t h_row_stride;
  const void* o_pre;  int64_t o_row_stride;
  const void* x_gate; int64_t x_gate_row_stride;
  void* out;          int64_t out_row_stride;
} hxm_mlstm_gates_args;

hxm_status hxm_mlstm_gate_prologue(const hxm_mlstm_gates_args* args, void* stream);
hxm_status hxm_mlstm_gate_epilogue(const hxm_mlstm_gates_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HXM_H_ */
