// Host-side plumbing of the block-scaled GEMM: the argument block handed from the C entry
// point to the per-instantiation launchers.
#pragma once

#include "../../include/quack_b200.h"
#include "qk_common.h"

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
