// mlstm_gates.cu — the element-wise gate work around the mLSTM recurrence
// (sm_100a), one HBM pass each:
//   prologue: log_i = i_pre, log_f = logsigmoid(f_pre)   (fp32 log-space gates)
//   epilogue: out = h * sigmoid(o_pre) * sigmoid(x_gate)
// Replaces i = exp(.), f = sigmoid(.), o = sigmoid(.) and h*o*sigmoid(x_gate)
// of mLSTMBlock.forward (hybrid_xmamba/layers/mlstm_block.py:117-119,138-141);
// the recurrence itself takes the gates in log space.
//
// A thread owns 8 consecutive elements of a row (16-byte loads for bf16,
// 16-byte stores); a ragged row tail or an unaligned row uses scalar elements.
#include "capi_internal.h"
#include "common.cuh"

namespace hxm {
namespace gates {

struct Params {
  int64_t rows;
  int dim;
  const void *ip, *fp;
  int64_t si, sf;
  float *li, *lf;
  int64_t sli, slf;
  const void *h, *op, *xg;
  int64_t sh, so, sx;
  void* out;
  int64_t sout;
};

// log(sigmoid(x)) = min(x, 0) - log1p(exp(-|x|)): the accurate form for fp32
// I/O, the MUFU form (absolute error ~1e-7) for bf16
template <bool ACC>
HXM_DEV float log_sigmoid(float x) {
  const float t = ACC ? log1pf(expf(-fabsf(x))) : kLn2 * lg2_approx(1.f + ex2_approx(-fabsf(x) * kLog2e));
  return fminf(x, 0.f) - t;
}

template <typename T>
HXM_DEV void load8(const T* p, bool vec, int n, float (&v)[8]) {
  if (sizeof(T) == 2 && vec) {
    const uint4 raw = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = to_f32<T>(e[j]);
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = j < n ? to_f32<T>(p[j]) : 0.f;
  }
}

// grid: x over 8-element vectors of a row, y (grid-stride) over rows
template <typename T>
__global__ void __launch_bounds__(256) prologue_kernel(const Params p) {
  constexpr bool ACC = sizeof(T) == 4;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= p.dim) return;
  const int n = min(8, p.dim - c);
  for (int64_t r = blockIdx.y; r < p.rows; r += gridDim.y) {
    const T* ip = static_cast<const T*>(p.ip) + r * p.si + c;
    const T* fp = static_cast<const T*>(p.fp) + r * p.sf + c;
    const bool vi = n == 8 && (reinterpret_cast<uintptr_t>(ip) % 16 == 0);
    const bool vf = n == 8 && (reinterpret_cast<uintptr_t>(fp) % 16 == 0);
    float a[8], f[8];
    load8<T>(ip, vi, n, a);
    load8<T>(fp, vf, n, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = log_sigmoid<ACC>(f[j]);
    float* li = p.li + r * p.sli + c;
    float* lf = p.lf + r * p.slf + c;
    if (n == 8 && reinterpret_cast<uintptr_t>(li) % 16 == 0 && reinterpret_cast<uintptr_t>(lf) % 16 == 0) {
      reinterpret_cast<float4*>(li)[0] = make_float4(a[0], a[1], a[2], a[3]);
      reinterpret_cast<float4*>(li)[1] = make_float4(a[4], a[5], a[6], a[7]);
      reinterpret_cast<float4*>(lf)[0] = make_float4(f[0], f[1], f[2], f[3]);
      reinterpret_cast<float4*>(lf)[1] = make_float4(f[4], f[5], f[6], f[7]);
    } else {
      for (int j = 0; j < n; ++j) {
        li[j] = a[j];
        lf[j] = f[j];
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) epilogue_kernel(const Params p) {
  constexpr bool ACC = sizeof(T) == 4;
  const int c = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (c >= p.dim) return;
  const int n = min(8, p.dim - c);
  for (int64_t r = blockIdx.y; r < p.rows; r += gridDim.y) {
    const T* hp = static_cast<const T*>(p.h) + r * p.sh + c;
    const T* op = static_cast<const T*>(p.op) + r * p.so + c;
    const T* xp = static_cast<const T*>(p.xg) + r * p.sx + c;
    T* outp = static_cast<T*>(p.out) + r * p.sout + c;
    auto al = [&](const void* q) { return n == 8 && reinterpret_cast<uintptr_t>(q) % 16 == 0; };
    float hv[8], ov[8], xv[8];
    load8<T>(hp, al(hp), n, hv);
    load8<T>(op, al(op), n, ov);
    load8<T>(xp, al(xp), n, xv);
    float y[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) y[j] = hv[j] * sigmoid<ACC>(ov[j]) * sigmoid<ACC>(xv[j]);
    if (sizeof(T) == 2 && al(outp)) {
      uint4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) e[j] = from_f32<T>(y[j]);
      *reinterpret_cast<uint4*>(outp) = raw;
    } else {
      for (int j = 0; j < n; ++j) outp[j] = from_f32<T>(y[j]);
    }
  }
}

static hxm_status fill(const hxm_mlstm_gates_args* a, Params& p, const char* who) {
  HXM_REQUIRE(a != nullptr, "%s: args is NULL", who);
  HXM_REQUIRE(a->struct_size == sizeof(hxm_mlstm_gates_args), "%s: struct_size %zu != %zu", who, a->struct_size,
              sizeof(hxm_mlstm_gates_args));
  HXM_REQUIRE(a->rows >= 0 && a->dim >= 1, "%s: bad rows=%lld dim=%d", who, (long long)a->rows, a->dim);
  HXM_REQUIRE(a->io_dtype == HXM_F32 || a->io_dtype == HXM_BF16, "%s: io_dtype must be f32 or bf16", who);
  p.rows = a->rows; p.dim = a->dim;
  p.ip = a->i_pre; p.fp = a->f_pre; p.si = a->i_row_stride; p.sf = a->f_row_stride;
  p.li = a->log_i; p.lf = a->log_f; p.sli = a->log_i_row_stride; p.slf = a->log_f_row_stride;
  p.h = a->h; p.op = a->o_pre; p.xg = a->x_gate; p.sh = a->h_row_stride; p.so = a->o_row_stride;
  p.sx = a->x_gate_row_stride; p.out = a->out; p.sout = a->out_row_stride;
  return HXM_OK;
}

static dim3 grid_for(const Params& p) {
  const int vec_blocks = (p.dim + 8 * 256 - 1) / (8 * 256);
  const int64_t rows = p.rows < 65535 ? p.rows : 65535;
  return dim3((unsigned)vec_blocks, (unsigned)(rows > 0 ? rows : 1));
}

}  // namespace gates
}  // namespace hxm

extern "C" hxm_status hxm_mlstm_gate_prologue(const hxm_mlstm_gates_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  gates::Params p{};
  hxm_status s = gates::fill(a, p, "hxm_mlstm_gate_prologue");
  if (s != HXM_OK) return s;
  if (p.rows == 0) return HXM_OK;
  HXM_REQUIRE(p.ip && p.fp && p.li && p.lf, "hxm_mlstm_gate_prologue: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->io_dtype == HXM_F32) gates::prologue_kernel<float><<<gates::grid_for(p), 256, 0, st>>>(p);
  else gates::prologue_kernel<__nv_bfloat16><<<gates::grid_for(p), 256, 0, st>>>(p);
  return check_launch("hxm_mlstm_gate_prologue");
}

extern "C" hxm_status hxm_mlstm_gate_epilogue(const hxm_mlstm_gates_args* a, void* stream) {
  using namespace hxm;
  clear_error();
  gates::Params p{};
  hxm_status s = gates::fill(a, p, "hxm_mlstm_gate_epilogue");
  if (s != HXM_OK) return s;
  if (p.rows == 0) return HXM_OK;
  HXM_REQUIRE(p.h && p.op && p.xg && p.out, "hxm_mlstm_gate_epilogue: NULL tensor pointer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->io_dtype == HXM_F32) gates::epilogue_kernel<float><<<gates::grid_for(p), 256, 0, st>>>(p);
  else gates::epilogue_kernel<__nv_bfloat16><<<gates::grid_for(p), 256, 0, st>>>(p);
  return check_launch("hxm_mlstm_gate_epilogue");
}
