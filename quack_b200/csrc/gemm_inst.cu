// Instantiations of the block-scaled GEMM kernel for one (QK_KIND, QK_QF) pair:
//   QK_KIND 0 = MXFP8 operands (kind::mxf8f6f4; E4M3 / E5M2 per operand), 1 = NVFP4 operands (kind::mxf4nvf4,
//           scale_vec::4X), 2 = MXFP4 operands (kind::mxf4nvf4, scale_vec::2X)
//   QK_QF   output format id: 0 = plain, QK_FMT_MXFP8_E4M3 (1), QK_FMT_NVFP4 (2) or QK_FMT_MXFP4 (4) re-quantised
// Compiled once per pair so that the pairs build in parallel.
#include "gemm_blockscaled.cuh"
#include "gemm_host.h"

#include <cstdlib>
#include <mutex>

#ifndef QK_KIND
#error "QK_KIND must be defined"
#endif
#ifndef QK_QF
#error "QK_QF must be defined"
#endif

namespace qk {
namespace {

constexpr int kMaxDevices = 64;

bool store_alignable(const void* p, long long ld_bytes) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) % 16 == 0) && (ld_bytes % 16 == 0);
}

template <int TILE_N, int CG, bool FEW_ROWS = false, bool PULL = false>
int launch_one(const GemmLaunch& l) {
  constexpr int KIND = QK_KIND;
  constexpr int QF = QK_QF;
  using C = GemmCfg<KIND, TILE_N, CG, FEW_ROWS, PULL>;
  const qk_gemm_args& a = *l.args;
  GemmParams p;
  memset(&p, 0, sizeof(p));
  const long long kbytes = KIND == 0 ? a.k : a.k / 2;
  const int vec = KIND == 1 ? 16 : 32;
  const long long sf_k = (a.k + vec - 1) / vec;
  const long long rk = (sf_k + 3) / 4;
  int rc;
  p.a_box_rows = (CG == 1 && a.m < C::TILE_M) ? static_cast<int>((a.m + 7) / 8 * 8) : C::TILE_M;
  if (FEW_ROWS && p.a_box_rows > C::A_ROWS_STORED)
    return qk_fail(QK_ERR_INVALID_ARG, "block-scaled GEMM: the few-rows kernel takes at most %d rows", C::A_ROWS_STORED);
  if ((rc = make_operand_map(&p.tm_a, a.a, a.m, kbytes, a.lda, p.a_box_rows)) != QK_OK) return rc;
  if ((rc = make_operand_map(&p.tm_b, a.b, a.n, kbytes, a.ldb, C::B_ROWS)) != QK_OK) return rc;
  if ((rc = make_scale_map(&p.tm_sfa, a.sfa, (a.m + 127) / 128, rk, a.sfa_stride_rm, a.sfa_stride_rk, C::AK, 1)) != QK_OK)
    return rc;
  if ((rc = make_scale_map(&p.tm_sfb, a.sfb, (a.n + 127) / 128, rk, a.sfb_stride_rm, a.sfb_stride_rk, C::AK, C::NB)) != QK_OK)
    return rc;
  p.M = a.m; p.N = a.n; p.K = a.k;
  p.tiles_m = (a.m + C::TILE_M * CG - 1) / (C::TILE_M * CG);
  p.tiles_n = (a.n + TILE_N - 1) / TILE_N;
  p.k_tiles = static_cast<int>((kbytes + C::KT_BYTES - 1) / C::KT_BYTES);
  p.group_m = 8;
  p.d = a.d; p.ldd = a.ldd; p.d_dtype = a.d_dtype; p.d_tma = 0; p.post_tma = 0;
  p.post = a.post; p.ldpost = a.ldpost; p.post_dtype = a.post ? a.post_dtype : a.d_dtype; p.act = a.activation;
  p.act_exact = a.exact_activation ? 1 : 0;
  if (KIND == 0) {
    const int fb = a.format_b ? a.format_b : a.format;
    p.idesc_elem_fmt = ((a.format == QK_FMT_MXFP8_E5M2 ? 1u : 0u) << 7) | ((fb == QK_FMT_MXFP8_E5M2 ? 1u : 0u) << 10);
  }
  if (!l.no_tma_store) {
    const bool gated = a.activation >= QK_ACT_GATED_FIRST;
    // element size and row width (in elements of the map) of an output holding `cols` logical columns
    auto build = [&](CUtensorMap* tm, int* flag, void* base, long long ld, int dtype, bool quant, int cols, int nv) -> int {
      if (base == nullptr) return QK_OK;
      int esize; long long ld_bytes, map_cols; int box_bytes;
      if (quant) {
        esize = 1;
        ld_bytes = ld;
        map_cols = qf_fp4(QF) ? cols / 2 : cols;
        box_bytes = qf_fp4(QF) ? nv / 2 : nv;
      } else {
        esize = dtype == QK_DT_F32 ? 4 : 2;
        ld_bytes = ld * esize;
        map_cols = cols;
        box_bytes = std::min(128, nv * esize);
      }
      // bulk tensor stores clip at the tensor bounds; keep to rows whose byte length is a
      // multiple of 16 so that the clip falls on a 16-byte boundary
      if (!store_alignable(base, ld_bytes) || (map_cols * esize) % 16 != 0) return QK_OK;
      const int rc2 = make_store_map(tm, base, esize, a.m, map_cols, ld_bytes, box_bytes);
      if (rc2 == QK_OK) *flag = 1;
      return rc2;
    };
    const bool quant_d = QF != QK_FMT_NONE && a.post == nullptr;
    if ((rc = build(&p.tm_d, &p.d_tma, a.d, a.ldd, a.d_dtype, quant_d, a.n, 64)) != QK_OK) return rc;
    if ((rc = build(&p.tm_post, &p.post_tma, a.post, a.ldpost, a.post_dtype, QF != QK_FMT_NONE, gated ? a.n / 2 : a.n,
                    gated ? 32 : 64)) != QK_OK)
      return rc;
  }
  p.bias = a.bias; p.bias_dtype = a.bias_dtype;
  p.alpha = a.alpha; p.alpha_dev = a.alpha_dev; p.alpha_dev2 = a.alpha_dev ? a.alpha_dev2 : nullptr;
  p.c = a.c; p.ldc = a.ldc; p.c_dtype = a.c_dtype; p.beta = a.beta; p.beta_dev = a.c ? a.beta_dev : nullptr;
  {
    const long long esz = a.c_dtype == QK_DT_F32 ? 4 : 2;
    p.c_vec_ok = (a.c != nullptr && (reinterpret_cast<uintptr_t>(a.c) & 15u) == 0 && (a.ldc * esz) % 16 == 0) ? 1 : 0;
  }
  p.sfd = static_cast<unsigned char*>(a.sfd); p.sfd_stride_rm = a.sfd_stride_rm;
  p.norm = a.norm_const; p.norm_dev = a.norm_const_dev;
  p.ag_flags = a.ag.flags; p.ag_epoch = a.ag.epoch;
  p.ag_num_shards = a.ag.num_shards; p.ag_first_shard = a.ag.first_shard; p.ag_num_chunks = a.ag.num_chunks;
  p.ag_pull = PULL ? a.ag.pull : nullptr;
  if (a.ag.flags != nullptr) {
    const int rows_per_shard = a.m / a.ag.num_shards;
    p.ag_tiles_m_per_shard = rows_per_shard / (C::TILE_M * CG);
  }
  p.timeout_ns = a.timeout_ns ? a.timeout_ns : 2000000000ull;
  p.status = a.status;
  p.vec_store_ok = l.vec_store_ok;
  p.prof = a.prof;
  {
    static const int pf_env = getenv("QK_PREFETCH_DIST") ? atoi(getenv("QK_PREFETCH_DIST")) : -1;
    p.prefetch_dist = pf_env >= 0 ? pf_env : 0;  // measured: prefetching ahead only adds L2 request traffic
  }
  p.clc = a.scheduler == QK_SCHED_CLC ? 1 : (a.scheduler == QK_SCHED_ARRIVAL ? 2 : 0);
  if (p.clc) p.prefetch_dist = 0;

  auto kernel = gemm_blockscaled_kernel<KIND, TILE_N, CG, QF, FEW_ROWS, PULL>;
  // The dynamic shared-memory limit is an attribute of the function in the CURRENT device's context: it is
  // set once per (instantiation, device), not once per process.
  {
    static std::mutex attr_mu;
    static bool attr_done[kMaxDevices] = {};
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return qk_fail(QK_ERR_CUDA, "block-scaled GEMM: cudaGetDevice failed");
    const int rc_attr = set_once_per_device(attr_mu, attr_done, dev, [&]() -> int {
      const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM_BYTES);
      if (e != cudaSuccess)
        return qk_fail(QK_ERR_CUDA, "cudaFuncSetAttribute(max dynamic smem %d) on device %d: %s", C::SMEM_BYTES, dev,
                       cudaGetErrorString(e));
      return QK_OK;
    });
    if (rc_attr != QK_OK) return rc_attr;
  }

  int sms = l.num_sms;
  if (a.max_ctas > 0) sms = std::min(sms, a.max_ctas);
  // split-K: a problem with fewer tiles than SMs streams its operands through too few CTAs to
  // cover the memory latency; splitting K puts every SM to work.  Needs caller workspace.
  p.split_k = 1;
  p.kt_per_split = p.k_tiles;
  {
    const int base_tiles = p.tiles_m * p.tiles_n;
    int want = a.split_k;
    if (want == 0) {   // automatic
      want = 1;
      // pays only when every split keeps a long K loop: publishing and summing the partials costs
      // several microseconds of dependent L2 round trips (measured: K = 4096 neutral, K = 14336
      // 1.6x faster at M <= 128)
      if (a.ag.flags == nullptr && a.workspace != nullptr && base_tiles * CG * 2 <= sms && p.k_tiles >= 48)
        want = std::min(std::min(sms / (base_tiles * CG), p.k_tiles / 24), 16);
    }
    if (want > 1) {
      if (a.ag.flags != nullptr) return qk_fail(QK_ERR_UNSUPPORTED, "block-scaled GEMM: split_k with the all-gather gate");
      want = std::min(want, p.k_tiles);
      const int per = (p.k_tiles + want - 1) / want;
      const int splits = (p.k_tiles + per - 1) / per;   // every split has at least one k-tile
      const size_t groups = static_cast<size_t>(base_tiles) * CG * 4;   // 32-row groups
      const size_t counter_bytes = (groups * sizeof(int) + 255) / 256 * 256;
      // one 8 KB block per (split, group, 64-column chunk)
      const size_t need = counter_bytes + static_cast<size_t>(splits) * groups * (TILE_N / 64) * 8192;
      if (a.workspace == nullptr || a.workspace_bytes < need) {
        if (a.split_k > 1)
          return qk_fail(QK_ERR_INVALID_ARG, "block-scaled GEMM: split_k=%d needs %zu bytes of zero-initialised workspace, got %llu",
                         a.split_k, need, a.workspace ? a.workspace_bytes : 0ull);
      } else if (splits > 1) {
        if (reinterpret_cast<uintptr_t>(a.workspace) & 15u)
          return qk_fail(QK_ERR_INVALID_ARG, "block-scaled GEMM: workspace must be 16-byte aligned");
        p.split_k = splits;
        p.kt_per_split = per;
        p.ws_counters = static_cast<int*>(a.workspace);
        p.ws_partials = reinterpret_cast<float*>(static_cast<unsigned char*>(a.workspace) + counter_bytes);
        p.ws_groups = static_cast<int>(groups);
      }
    }
  }
  const int num_tiles = p.tiles_m * p.tiles_n * p.split_k;
  int clusters = std::min(num_tiles, sms / CG);
  if (clusters < 1) clusters = 1;
  // dynamic scheduler: one cluster per tile; the clusters that get SMs first cancel the launch of
  // the others and compute their tiles
  if (p.clc == 1) clusters = num_tiles;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(static_cast<unsigned>(clusters * CG), 1, 1);
  cfg.blockDim = dim3(C::NUM_THREADS, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = static_cast<cudaStream_t>(a.stream);
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // the kernel waits (griddepcontrol.wait) before its first global access, so it may be scheduled
  // while the previous kernel of the stream is still running
  static const bool no_pdl = getenv("QK_NO_PDL") != nullptr;
  if (!no_pdl) {
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.numAttrs = 2;
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  qk_count_launch();
  if (e != cudaSuccess) return qk_fail(QK_ERR_CUDA, "block-scaled GEMM launch: %s", cudaGetErrorString(e));
  return QK_OK;
}

}  // namespace

#define QK_CAT_(a, b, c, d) a##b##c##d
#define QK_CAT(a, b, c, d) QK_CAT_(a, b, c, d)
int QK_CAT(launch_gemm_k, QK_KIND, _q, QK_QF)(const GemmLaunch& l) {
  const int key = l.tile_n * 10 + l.cta_group;
  if (l.args->ag.flags != nullptr && l.args->ag.pull != nullptr) {   // in-kernel transport: one more warp per CTA
    if (key == 2562) return launch_one<256, 2, false, true>(l);
    return qk_fail(QK_ERR_UNSUPPORTED, "block-scaled GEMM: the in-kernel all-gather transport needs tile_n=256, cta_group=2");
  }
  if (l.cta_group == 1 && l.args->m <= 32) {   // few rows: the deep-pipeline variants
    switch (key) {
      case 641: return launch_one<64, 1, true>(l);
      case 1281: return launch_one<128, 1, true>(l);
      case 2561: return launch_one<256, 1, true>(l);
      default: break;
    }
  }
  switch (key) {
    case 641: return launch_one<64, 1>(l);
    case 1281: return launch_one<128, 1>(l);
    case 2561: return launch_one<256, 1>(l);
    case 1282: return launch_one<128, 2>(l);
    case 1922: return launch_one<192, 2>(l);
    case 2562: return launch_one<256, 2>(l);
    default:
      return qk_fail(QK_ERR_UNSUPPORTED, "block-scaled GEMM: no kernel for tile_n=%d cta_group=%d", l.tile_n, l.cta_group);
  }
}

}  // namespace qk
