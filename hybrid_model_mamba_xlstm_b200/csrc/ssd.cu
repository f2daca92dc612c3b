// ssd.cu — C ABI of the Mamba-2 SSD chunked scan (ngroups = 1) on tcgen05.
//
// The reference has no SSD kernel; the recurrence is its Euler selective scan
// (hybrid_xmamba/kernels/selective_scan/scan_interface.py:132-150) with
// channel (head, p), per-head A and dt, and B, C shared by all heads.  It runs
// the chunkwise kernel of chunk_tc.cuh: the state (dstate x headdim) in TMEM,
// C B^T / P x / C state / state update on the tensor cores.
#include "chunk_tc.cuh"
#include "tma_host.h"

using namespace hxm;
using namespace hxm::chunk;

extern "C" size_t hxm_ssd_workspace_size(const hxm_ssd_args*) { return 0; }

template <int DK>
static hxm_status launch_ssd(const hxm_ssd_args* a, cudaStream_t st) {
  const int B = a->batch, L = a->seqlen, H = a->heads, P = a->headdim;
  CUtensorMap mc, mb, mx;
  const uint64_t dn[4] = {(uint64_t)DK, (uint64_t)L, 1, (uint64_t)B};
  const uint64_t sn[3] = {(uint64_t)DK * 2, (uint64_t)L * DK * 2, (uint64_t)L * DK * 2};
  const uint64_t dx[4] = {(uint64_t)P, (uint64_t)L, (uint64_t)H, (uint64_t)B};
  const uint64_t sx[3] = {(uint64_t)H * P * 2, (uint64_t)P * 2, (uint64_t)L * H * P * 2};
  hxm_status s;
  if ((s = make_map_bf16_4d(&mc, a->C, dn, sn, "ssd C")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mb, a->B, dn, sn, "ssd B")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mx, a->x, dx, sx, "ssd x")) != HXM_OK) return s;
  Params cp{};
  cp.batch = B; cp.heads = H; cp.seqlen = L; cp.dv = P;
  cp.g0 = a->dt; cp.sg0[0] = (int64_t)L * H; cp.sg0[1] = 1; cp.sg0[2] = H;
  cp.A = a->A; cp.dt_bias = a->dt_bias; cp.dt_softplus = a->dt_softplus; cp.Dskip = a->D;
  cp.x = static_cast<const __nv_bfloat16*>(a->x);
  cp.sx[0] = (int64_t)L * H * P; cp.sx[1] = P; cp.sx[2] = (int64_t)H * P;
  cp.out = static_cast<__nv_bfloat16*>(a->y);
  cp.so[0] = cp.sx[0]; cp.so[1] = cp.sx[1]; cp.so[2] = cp.sx[2];
  cp.C0 = a->h0; cp.CT = a->hT; cp.state_t = 1;
  cp.error_flag = a->error_flag;
  cp.wait_limit = a->wait_limit_cycles != 0 ? a->wait_limit_cycles : 4000000000ll;
  const size_t smem = Layout<DK>::kBytes + 1024;
  auto kern = chunk_tc_kernel<DK, kSsd>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((P + kDV - 1) / kDV, H, B);
  kern<<<grid, kThreads, smem, st>>>(mc, mb, mx, cp);
  return check_launch("hxm_ssd_chunk_scan_fwd");
}

extern "C" hxm_status hxm_ssd_chunk_scan_fwd(const hxm_ssd_args* a, void* stream) {
  clear_error();
  HXM_REQUIRE(a != nullptr, "hxm_ssd_chunk_scan_fwd: args is NULL");
  HXM_REQUIRE(a->struct_size == sizeof(hxm_ssd_args), "hxm_ssd_chunk_scan_fwd: struct_size %zu != %zu",
              a->struct_size, sizeof(hxm_ssd_args));
  HXM_REQUIRE(a->batch >= 0 && a->seqlen >= 0 && a->heads >= 0 && a->headdim >= 1 && a->dstate >= 1,
              "hxm_ssd_chunk_scan_fwd: bad dims");
  // the kernel tiles time in 128-step chunks (the chunkwise result does not depend on the length);
  // other lengths are refused rather than silently replaced
  HXM_REQUIRE_SUPPORTED(a->chunk == 0 || a->chunk == kC,
                        "hxm_ssd_chunk_scan_fwd: chunk %d unsupported (the kernel runs %d-step chunks; pass 0 or %d)",
                        a->chunk, kC, kC);
  HXM_REQUIRE(a->io_dtype == HXM_BF16, "hxm_ssd_chunk_scan_fwd: io_dtype must be bf16");
  HXM_REQUIRE_SUPPORTED(a->dstate == 128 || a->dstate == 256, "hxm_ssd_chunk_scan_fwd: dstate %d (128 or 256 supported)",
                        a->dstate);
  HXM_REQUIRE_SUPPORTED(a->headdim % 32 == 0, "hxm_ssd_chunk_scan_fwd: headdim %d must be a multiple of 32", a->headdim);
  if (a->batch == 0 || a->heads == 0) return HXM_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (a->seqlen == 0) {
    if (a->hT) {
      const size_t bytes = sizeof(float) * (size_t)a->batch * a->heads * a->headdim * a->dstate;
      if (a->h0) HXM_CUDA_TRY(cudaMemcpyAsync(a->hT, a->h0, bytes, cudaMemcpyDeviceToDevice, st));
      else HXM_CUDA_TRY(cudaMemsetAsync(a->hT, 0, bytes, st));
    }
    return HXM_OK;
  }
  HXM_REQUIRE(a->x && a->dt && a->A && a->B && a->C && a->y, "hxm_ssd_chunk_scan_fwd: NULL tensor pointer");
  return a->dstate == 128 ? launch_ssd<128>(a, st) : launch_ssd<256>(a, st);
}
