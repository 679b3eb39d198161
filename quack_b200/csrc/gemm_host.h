// Host-side plumbing of the block-scaled GEMM: the argument block handed from the C entry
// point to the per-instantiation launchers.
#pragma once

#include "../../include/quack_b200.h"
#include "qk_common.h"

#include <cuda.h>

#include <mutex>

namespace qk {

// Runs `fn` the first time it is called for device index `dev` (0 <= dev < N) and remembers success; a
// failure is returned and retried by the next call.  `done` and `mu` belong to the caller (one pair per
// thing that has to happen once per device).  Devices outside the table run `fn` every time.
template <int N, typename Fn>
int set_once_per_device(std::mutex& mu, bool (&done)[N], int dev, Fn&& fn) {
  if (dev < 0 || dev >= N) return fn();
  std::lock_guard<std::mutex> lock(mu);
  if (done[dev]) return QK_OK;
  const int rc = fn();
  if (rc == QK_OK) done[dev] = true;
  return rc;
}

// Tensor maps (TMA descriptors) of the GEMM, built through cuTensorMapEncodeTiled and kept in a small
// process-wide cache keyed by everything that goes into one (address, extents, strides, box, element type,
// swizzle): a descriptor depends on nothing else, so a hit is valid for as long as the key repeats, and a
// serving loop that calls with the same buffers pays the driver call once.
//   operand: K-major (rows, kbytes) bytes with row pitch ld; box = 128 bytes x box_rows, 128-byte swizzle
//   scales:  blocked scale factors, (rm, rk) atoms of 512 bytes = 128 uint32; box = (128, box_k, box_mn)
//   store:   output matrix for the staged bulk store; box = box_bytes x 32 rows, swizzle mode = box width
int make_operand_map(CUtensorMap* tm, const void* base, long long rows, long long kbytes, long long ld, int box_rows);
int make_scale_map(CUtensorMap* tm, const void* base, long long rm, long long rk, long long stride_rm, long long stride_rk,
                   int box_k, int box_mn);
int make_store_map(CUtensorMap* tm, const void* base, int esize, long long rows, long long cols, long long ld_bytes,
                   int box_bytes);
// (hits, misses) of the cache since the library was loaded
void tensor_map_cache_stats(long long* hits, long long* misses);

struct GemmLaunch {
  const qk_gemm_args* args;
  int tile_n;
  int cta_group;
  int num_sms;
  int vec_store_ok;
  int no_tma_store;  // debugging aid: force the register -> global store path
};

// One launcher per (operand kind, output format) pair; each covers every tile_n / CTA group it was
// instantiated for and returns QK_ERR_UNSUPPORTED for the rest.  Kinds: 0 MXFP8, 1 NVFP4, 2 MXFP4; the
// output index is the QK_FMT_* id of the re-quantised output (0 = plain).
#define QK_DECLARE_LAUNCHERS(K)                   \
  int launch_gemm_k##K##_q0(const GemmLaunch& l); \
  int launch_gemm_k##K##_q1(const GemmLaunch& l); \
  int launch_gemm_k##K##_q2(const GemmLaunch& l); \
  int launch_gemm_k##K##_q4(const GemmLaunch& l);
QK_DECLARE_LAUNCHERS(0)
QK_DECLARE_LAUNCHERS(1)
QK_DECLARE_LAUNCHERS(2)
#undef QK_DECLARE_LAUNCHERS

}  // namespace qk
