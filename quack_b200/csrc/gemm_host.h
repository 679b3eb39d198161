// Host-side plumbing of the block-scaled GEMM: the argument block handed from the C entry
// point to the per-instantiation launchers.
#pragma once

#include "../../include/quack_b200.h"
#include "qk_common.h"

namespace qk {

struct GemmLaunch {
  const qk_gemm_args* args;
  int tile_n;
  int cta_group;
  int num_sms;
  int vec_store_ok;
  int no_tma_store;  // debugging aid: force the register -> global store path
};

// One launcher per (operand kind, output quantisation) pair; each covers every tile_n / CTA
// group it was instantiated for and returns QK_ERR_UNSUPPORTED for the rest.
int launch_gemm_k0_q0(const GemmLaunch& l);
int launch_gemm_k0_q1(const GemmLaunch& l);
int launch_gemm_k0_q2(const GemmLaunch& l);
int launch_gemm_k1_q0(const GemmLaunch& l);
int launch_gemm_k1_q1(const GemmLaunch& l);
int launch_gemm_k1_q2(const GemmLaunch& l);

}  // namespace qk
