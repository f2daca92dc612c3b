// mlstm_tc.cu — launch of the tcgen05 chunkwise mLSTM (per-head gates, bf16).
#include "chunk_tc.cuh"
#include "mlstm.h"
#include "tma_host.h"

namespace hxm {
namespace mlstm {

static bool tc_shape_ok(const Params& p) {
  if (p.io_dtype != HXM_BF16 || p.gate_mode != 0) return false;
  if (p.dqk != 128 && p.dqk != 256) return false;
  if (p.dv % 32 != 0) return false;
  auto ok = [](int64_t s) { return s % 8 == 0; };
  return ok(p.sq[0]) && ok(p.sq[1]) && ok(p.sk[0]) && ok(p.sk[1]) && ok(p.sv[0]) && ok(p.sv[1]) &&
         ok(p.tq) && ok(p.tk) && ok(p.tv) && ok(p.th) &&
         reinterpret_cast<uintptr_t>(p.q) % 16 == 0 && reinterpret_cast<uintptr_t>(p.k) % 16 == 0 &&
         reinterpret_cast<uintptr_t>(p.v) % 16 == 0 && reinterpret_cast<uintptr_t>(p.h) % 16 == 0 &&
         p.sh[0] % 8 == 0 && p.sh[1] % 8 == 0 && p.seqlen > 0;
}

size_t chunkwise_tc_workspace(const Params& p) { return tc_shape_ok(p) ? 0 : (size_t)-1; }

template <int DK>
static hxm_status launch_dk(const Params& p, cudaStream_t st) {
  using namespace hxm::chunk;
  CUtensorMap mq, mk, mv;
  const uint64_t dq[4] = {(uint64_t)DK, (uint64_t)p.seqlen, (uint64_t)p.heads, (uint64_t)p.batch};
  const uint64_t sq[3] = {(uint64_t)p.tq * 2, (uint64_t)p.sq[1] * 2, (uint64_t)p.sq[0] * 2};
  const uint64_t sk[3] = {(uint64_t)p.tk * 2, (uint64_t)p.sk[1] * 2, (uint64_t)p.sk[0] * 2};
  const uint64_t dvd[4] = {(uint64_t)p.dv, (uint64_t)p.seqlen, (uint64_t)p.heads, (uint64_t)p.batch};
  const uint64_t sv[3] = {(uint64_t)p.tv * 2, (uint64_t)p.sv[1] * 2, (uint64_t)p.sv[0] * 2};
  hxm_status s;
  if ((s = make_map_bf16_4d(&mq, p.q, dq, sq, "mlstm q")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mk, p.k, dq, sk, "mlstm k")) != HXM_OK) return s;
  if ((s = make_map_bf16_4d(&mv, p.v, dvd, sv, "mlstm v")) != HXM_OK) return s;
  chunk::Params cp{};
  cp.batch = p.batch; cp.heads = p.heads; cp.seqlen = p.seqlen; cp.dv = p.dv;
  cp.g0 = p.log_i; cp.sg0[0] = p.si[0]; cp.sg0[1] = p.si[1]; cp.sg0[2] = p.ti;
  cp.g1 = p.log_f; cp.sg1[0] = p.sf[0]; cp.sg1[1] = p.sf[1]; cp.sg1[2] = p.tf;
  cp.out = static_cast<__nv_bfloat16*>(p.h);
  cp.so[0] = p.sh[0]; cp.so[1] = p.sh[1]; cp.so[2] = p.th;
  cp.C0 = p.C0; cp.n0 = p.n0; cp.m0 = p.m0; cp.CT = p.CT; cp.nT = p.nT; cp.mT = p.mT;
  cp.state_t = 0;
  cp.error_flag = p.error_flag;
  cp.wait_limit = p.wait_limit;
  const size_t smem = Layout<DK>::kBytes + 1024;
  auto kern = chunk_tc_kernel<DK, kMlstm>;
  HXM_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  dim3 grid((p.dv + kDV - 1) / kDV, p.heads, p.batch);
  kern<<<grid, kThreads, smem, st>>>(mq, mk, mv, cp);
  return check_launch("hxm_mlstm_chunkwise_fwd (tcgen05)");
}

hxm_status launch_chunkwise_tc(const Params& p, cudaStream_t st) {
  if (p.dqk == 128) return launch_dk<128>(p, st);
  return launch_dk<256>(p, st);
}

}  // namespace mlstm
}  // namespace hxm
