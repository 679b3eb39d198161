// C entry point of the block-scaled GEMM: argument validation, configuration choice, dispatch.
#include "gemm_host.h"

#include <cstdlib>
#include <mutex>

using namespace qk;

namespace {

int device_sm_count() {
  static int sms[64];
  static std::once_flag once;
  std::call_once(once, [] { for (int& s : sms) s = 0; });
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (sms[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess) sms[dev] = v;
  }
  return sms[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" int qk_gemm_blockscaled(const qk_gemm_args* a) {
  if (a == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: null argument block");
  // MMA kind of the operand pair (quack/blockscaled/operand.py:418-483): the two MXFP8 element types mix
  // freely under kind::mxf8f6f4; the 4-bit formats pair only with themselves
  const int fmt_b = a->format_b ? a->format_b : a->format;
  auto is_fp8 = [](int f) { return f == QK_FMT_MXFP8_E4M3 || f == QK_FMT_MXFP8_E5M2; };
  int kind;
  if (is_fp8(a->format) && is_fp8(fmt_b)) kind = 0;
  else if (a->format == QK_FMT_NVFP4 && fmt_b == QK_FMT_NVFP4) kind = 1;
  else if (a->format == QK_FMT_MXFP4 && fmt_b == QK_FMT_MXFP4) kind = 2;
  else
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled: no MMA kind for operand formats %d x %d (MXFP8 E4M3 / E5M2 "
                   "mix freely; MXFP4 and NVFP4 pair only with themselves)", a->format, fmt_b);
  if (a->m < 0 || a->n < 0 || a->k < 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: negative extent");
  if (a->m == 0 || a->n == 0) return QK_OK;
  if (a->k == 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: K == 0 is handled by the caller");
  if (a->k % 32 != 0) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: K (%d) must be a multiple of 32", a->k);
  if (!a->a || !a->b || !a->sfa || !a->sfb) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: null operand pointer");
  if (!aligned16(a->a) || !aligned16(a->b) || (a->lda % 16) || (a->ldb % 16))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: A/B base and row pitch must be 16-byte aligned");
  const long long kbytes = kind == 0 ? a->k : a->k / 2;
  if (a->lda < kbytes || a->ldb < kbytes) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: row pitch smaller than a row");
  if (!aligned16(a->sfa) || !aligned16(a->sfb) || (a->sfa_stride_rm % 512) || (a->sfa_stride_rk % 512) ||
      (a->sfb_stride_rm % 512) || (a->sfb_stride_rk % 512))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: scale atoms must be 512-byte granular and 16-byte aligned");
  if (a->status == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: status buffer is required");
  if (a->d == nullptr && a->post == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: no output");
  if (a->c != nullptr && (a->c_dtype < QK_DT_BF16 || a->c_dtype > QK_DT_F32 || a->ldc < a->n))
    return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: bad residual operand (dtype %d, ldc %lld)", a->c_dtype, a->ldc);
  const bool gated = a->activation >= QK_ACT_GATED_FIRST;
  if (a->post == nullptr && a->activation != QK_ACT_NONE)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: an activation needs the post output");
  if (gated && (a->n % 2)) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: gated activation needs even N");
  const int qf = a->out_format;
  if (qf != QK_FMT_NONE && qf != QK_FMT_MXFP8_E4M3 && qf != QK_FMT_NVFP4 && qf != QK_FMT_MXFP4)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled: output format %d has no quantising epilogue "
                   "(MXFP8_E4M3, MXFP4, NVFP4)", qf);
  if (qf != QK_FMT_NONE) {
    if (a->sfd == nullptr) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: quantised output needs sfd");
    if (a->sfd_stride_rm % 512) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: sfd stride must be 512-byte granular");
    const int n_out = gated ? a->n / 2 : a->n;
    const int need = (qf == QK_FMT_NVFP4 || qf == QK_FMT_MXFP4) ? 32 : 16;
    if (n_out % need) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: quantised output needs N %% %d == 0", need);
  }
  if (a->ag.flags != nullptr) {
    if (a->ag.epoch == nullptr || a->ag.num_shards < 1 || a->ag.num_chunks < 1 || a->ag.first_shard < 0 ||
        a->ag.first_shard >= a->ag.num_shards)
      return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: bad all-gather arguments");
    if (a->m % a->ag.num_shards) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: M must divide evenly into shards");
    if (a->ag.pull != nullptr) {
      // (pull mode: one shard per rank, at most QK_AG_MAX_RANKS; multicast mode: ranks x chunks shards)
      if (a->ag.num_chunks != 1 || a->ag.num_shards > 32 || (a->m / a->ag.num_shards) % 256)
        return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: the in-kernel all-gather transport needs one chunk per shard, "
                       "at most 32 shards and shard rows that are a multiple of 256");
      if ((a->tile_n != 0 && a->tile_n != 256) || (a->cta_group != 0 && a->cta_group != 2))
        return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled: the in-kernel all-gather transport runs on 256-wide CTA-pair tiles");
    }
  }

  if (a->scheduler != QK_SCHED_STATIC && a->scheduler != QK_SCHED_CLC && a->scheduler != QK_SCHED_ARRIVAL)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: scheduler must be QK_SCHED_STATIC, QK_SCHED_CLC or QK_SCHED_ARRIVAL");
  if (a->scheduler == QK_SCHED_ARRIVAL &&
      (a->ag.flags == nullptr || a->ag.num_chunks != 1 || a->ag.num_shards > 32))
    return qk_fail(QK_ERR_INVALID_ARG,
                   "qk_gemm_blockscaled: the arrival-order scheduler needs all-gather arguments with one chunk per shard and at most 32 shards");
  if (a->scheduler == QK_SCHED_CLC && a->prof != nullptr)
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled: role counters (prof) need the static scheduler");
  if (a->scheduler == QK_SCHED_CLC && a->max_ctas > 0)
    return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: max_ctas needs the static scheduler (the dynamic one fills every SM)");
  const int sms = device_sm_count();
  if (sms <= 0) return qk_fail(QK_ERR_CUDA, "qk_gemm_blockscaled: cannot query the device");

  // configuration: large problems use 256-row tiles across a CTA pair, small ones 128x128
  // (rule of quack/gemm_config.py:308-314); explicit requests win
  int cg = a->cta_group, tile_n = a->tile_n;
  if (a->ag.flags != nullptr && a->ag.pull != nullptr) { cg = 2; tile_n = 256; }
  if (cg == 0 && tile_n == 0) {
    // Pick the compiled tile shape with the smallest modelled main-loop time:
    //   (tiles each cluster works through) x (time of one k-tile of that shape).
    // The per-k-tile costs are measured on B200 (microseconds at K = 4096 bytes, one wave):
    // narrow tiles are bound by the issue of their MMA / scale-copy instructions (~0.3 us per
    // k-tile whatever the width), 256-wide pair tiles by the tensor pipe.  The count term is
    // what matters: it removes partial waves (e.g. 192-wide tiles for N = 6144, M = 1024) and
    // gives few-row problems enough CTAs to stream the weights.
    struct Cand { int tile_n, cg; double cost; };
    static const Cand cands[] = {{256, 2, 0.456}, {192, 2, 0.390}, {128, 2, 0.360}, {256, 1, 0.520}, {128, 1, 0.300}, {64, 1, 0.270}};
    double best = 0;
    for (const Cand& c : cands) {
      if (a->ag.flags != nullptr && (a->m / a->ag.num_shards) % (128 * c.cg * a->ag.num_chunks)) continue;
      if (c.cg == 2 && a->m <= 128) continue;   // half of every pair would be padding
      const long long tiles = ((a->m + 128LL * c.cg - 1) / (128 * c.cg)) * ((a->n + c.tile_n - 1) / c.tile_n);
      int clusters = sms / c.cg;
      if (a->max_ctas > 0) clusters = std::max(1, std::min(sms, a->max_ctas) / c.cg);
      const double t = static_cast<double>((tiles + clusters - 1) / clusters) * c.cost;
      if (cg == 0 || t < best * 0.999) {   // ties keep the earlier (larger) shape
        best = t;
        cg = c.cg;
        tile_n = c.tile_n;
      }
    }
    if (cg == 0) { cg = 1; tile_n = 128; }
    // Long K with few tiles is split over K by the launcher; there 128-wide tiles with twice the splits beat
    // 64-wide ones (down-projection M <= 128: 20.2 vs 22.4 us): half the partial-sum traffic per weight byte.
    const long long kbytes_model = kbytes;
    if (cg == 1 && tile_n == 64 && a->workspace != nullptr && a->split_k == 0 && a->ag.flags == nullptr &&
        kbytes_model / 128 >= 96 && ((a->m + 127) / 128) * ((a->n + 127) / 128) * 2 <= sms)
      tile_n = 128;
  }
  if (cg == 0) cg = (a->m >= 512 && a->n >= 128) ? 2 : 1;
  if (tile_n == 0) tile_n = (a->m >= 512 && a->n >= 256 && cg == 2) ? 256 : 128;
  if (cg != 1 && cg != 2) return qk_fail(QK_ERR_INVALID_ARG, "qk_gemm_blockscaled: cta_group must be 0, 1 or 2");
  if (tile_n % 64 != 0 && (a->post != nullptr || qf != QK_FMT_NONE))
    return qk_fail(QK_ERR_UNSUPPORTED, "qk_gemm_blockscaled: tile_n=%d supports plain outputs only", tile_n);
  if (a->ag.flags != nullptr) {
    const int rows_per_shard = a->m / a->ag.num_shards;
    if (rows_per_shard % (128 * cg * a->ag.num_chunks))
      return qk_fail(QK_ERR_INVALID_ARG,
                     "qk_gemm_blockscaled: shard rows (%d) must be a multiple of tile rows x chunks (%d)",
                     rows_per_shard, 128 * cg * a->ag.num_chunks);
  }

  // 16-byte vector stores need aligned bases and pitches; otherwise the epilogue stores scalars
  int vec_ok = 1;
  auto chk = [&](const void* p, long long ld_elems, int dtype, bool quant_codes) {
    if (p == nullptr) return;
    const long long esz = quant_codes ? 1 : (dtype == QK_DT_F32 ? 4 : 2);
    if (!aligned16(p) || ((ld_elems * esz) % 16)) vec_ok = 0;
  };
  chk(a->d, a->ldd, a->d_dtype, qf != QK_FMT_NONE && a->post == nullptr);
  chk(a->post, a->ldpost, a->post_dtype, qf != QK_FMT_NONE);

  static const bool no_tma = getenv("QK_NO_TMA_STORE") != nullptr;
  GemmLaunch l{a, tile_n, cg, sms, vec_ok, no_tma ? 1 : 0};
  typedef int (*Launcher)(const GemmLaunch&);
  static const Launcher table[3][4] = {
      {launch_gemm_k0_q0, launch_gemm_k0_q1, launch_gemm_k0_q2, launch_gemm_k0_q4},
      {launch_gemm_k1_q0, launch_gemm_k1_q1, launch_gemm_k1_q2, launch_gemm_k1_q4},
      {launch_gemm_k2_q0, launch_gemm_k2_q1, launch_gemm_k2_q2, launch_gemm_k2_q4}};
  const int qi = qf == QK_FMT_NONE ? 0 : qf == QK_FMT_MXFP8_E4M3 ? 1 : qf == QK_FMT_NVFP4 ? 2 : 3;
  return table[kind][qi](l);
}
