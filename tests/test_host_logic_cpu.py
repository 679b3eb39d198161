"""Host-side logic that needs no GPU: the torch.library op registrations, and the once-per-device
bookkeeping of the C++ launcher (compiled with g++ against the library's own header)."""

import os
import subprocess
import sys
import textwrap

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_custom_ops_are_registered_with_the_reference_names():
    from quack_b200 import _torch_ops
    ns = getattr(torch.ops, _torch_ops.NAMESPACE)
    for name in ("gemm_out", "gemm_quant_out", "gemm_add_out", "gemm_add_inplace", "gemm_act_out"):
        schema = str(getattr(ns, name).default._schema)
        assert "Tensor A, Tensor B" in schema and "SFA" in schema and "bs_format_a" in schema, schema
    s = str(ns.gemm_quant_out.default._schema)
    assert "Tensor(a2!) out" in s and "Tensor(a3!) SFD" in s and "str bs_format_d" in s       # both outputs are mutated
    # e8m0 scale factors and 4-bit codes cross the boundary as uint8 views, bytes unchanged
    sf = torch.zeros(1, 1, 32, 4, 4, dtype=torch.uint8).view(torch.float8_e8m0fnu)
    assert _torch_ops.encode(sf).dtype == torch.uint8 and _torch_ops.encode(sf).data_ptr() == sf.data_ptr()
    assert _torch_ops.encode(torch.zeros(4, dtype=torch.float8_e4m3fn)).dtype == torch.float8_e4m3fn


def test_once_per_device_bookkeeping(tmp_path):
    """The kernel's dynamic shared-memory attribute belongs to a device's context, so it is set once per
    (kernel, device), not once per process: the helper that keeps that book is driven here with injected
    device indices (a second device, an index outside the table, a failure that must be retried)."""
    src = tmp_path / "once.cpp"
    src.write_text(textwrap.dedent('''
        #include "quack_b200/csrc/gemm_host.h"
        #include <cstdio>
        int qk_fail(int code, const char*, ...) { return code; }
        int main() {
          static std::mutex mu;
          static bool done[4] = {};
          int calls = 0;
          auto ok = [&]() { ++calls; return QK_OK; };
          int fails_left = 1;
          auto flaky = [&]() { ++calls; return fails_left-- > 0 ? QK_ERR_CUDA : QK_OK; };
          if (qk::set_once_per_device(mu, done, 0, ok) != QK_OK || calls != 1) return 1;
          if (qk::set_once_per_device(mu, done, 0, ok) != QK_OK || calls != 1) return 2;   // remembered
          if (qk::set_once_per_device(mu, done, 1, ok) != QK_OK || calls != 2) return 3;   // a second device runs it again
          if (qk::set_once_per_device(mu, done, 2, flaky) != QK_ERR_CUDA || calls != 3) return 4;
          if (qk::set_once_per_device(mu, done, 2, flaky) != QK_OK || calls != 4) return 5; // a failure is not remembered
          if (qk::set_once_per_device(mu, done, 2, flaky) != QK_OK || calls != 4) return 6;
          if (qk::set_once_per_device(mu, done, 7, ok) != QK_OK || calls != 5) return 7;   // outside the table: every time
          if (qk::set_once_per_device(mu, done, 7, ok) != QK_OK || calls != 6) return 8;
          if (qk::set_once_per_device(mu, done, -1, ok) != QK_OK || calls != 7) return 9;
          std::puts("ONCE_OK");
          return 0;
        }
    '''))
    exe = tmp_path / "once"
    cuda_inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
    subprocess.run(["g++", "-std=c++17", "-I", ROOT, "-I", cuda_inc, str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True)
    assert r.returncode == 0 and "ONCE_OK" in r.stdout, (r.returncode, r.stdout, r.stderr)


def test_ctypes_mirrors_match_the_c_header(tmp_path):
    """The Python side hands the library ctypes mirrors of the header's structs: sizes and the offsets of the
    fields added last must agree with what a C compiler makes of ``include/quack_b200.h``."""
    import ctypes as C
    from quack_b200 import _lib
    src = tmp_path / "layout.c"
    src.write_text(textwrap.dedent('''
        #include "include/quack_b200.h"
        #include <stddef.h>
        #include <stdio.h>
        int main(void) {
          printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", sizeof(qk_ag_pull_args), offsetof(qk_ag_pull_args, peer_base),
                 offsetof(qk_ag_pull_args, peer_drained), offsetof(qk_ag_pull_args, flags_rw), sizeof(qk_ag_args),
                 offsetof(qk_ag_args, pull), sizeof(qk_gemm_args), offsetof(qk_gemm_args, ag));
          return 0;
        }
    '''))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", ROOT, str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    P, A, G = _lib.AgPullArgs, _lib.AgArgs, _lib.GemmArgs
    want = [C.sizeof(P), P.peer_base.offset, P.peer_drained.offset, P.flags_rw.offset, C.sizeof(A), A.pull.offset,
            C.sizeof(G), G.ag.offset]
    assert got == want
