"""The tcgen05 shared-memory and instruction descriptors of webgpu_b200/csrc/umma.cuh
against an independent encoding: CUTLASS's cute::UMMA::SmemDescriptor and
InstrDescriptor bitfields (compiled as host code with nvcc, no GPU needed).
Skipped when nvcc or a CUTLASS header tree is not available."""
import glob
import os
import shutil
import subprocess
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r'''
#include <cstdio>
#include <cute/arch/mma_sm100_desc.hpp>
#include "webgpu_b200/csrc/umma.cuh"
int main() {
  int bad = 0;
  const unsigned addrs[] = {0u, 16u, 1024u, 37888u, 152576u, 209392u, 232432u};
  const unsigned offs[] = {16u, 128u, 256u, 1024u, 4096u, 16384u};
  for (unsigned addr : addrs)
    for (unsigned lbo : offs)
      for (unsigned sbo : offs) {
        cute::UMMA::SmemDescriptor d;
        d.start_address_ = addr >> 4;
        d.leading_byte_offset_ = lbo >> 4;
        d.stride_byte_offset_ = sbo >> 4;
        d.version_ = 1;
        d.base_offset_ = 0;
        d.lbo_mode_ = 0;
        d.layout_type_ = 0;
        if ((uint64_t)d != wgd::tc::sdesc(addr, lbo, sbo)) { bad++; printf("sdesc %u %u %u\n", addr, lbo, sbo); }
      }
  for (int m : {64, 128})
    for (int n = 16; n <= 256; n += 16) {
      cute::UMMA::InstrDescriptor d;
      d.desc_ = 0;
      d.c_format_ = 1;   // F32
      d.a_format_ = 0;   // F16
      d.b_format_ = 0;
      d.a_major_ = 0;    // K-major
      d.b_major_ = 0;
      d.n_dim_ = n >> 3;
      d.m_dim_ = m >> 4;
      if ((uint32_t)d != wgd::tc::idesc_f16_f32(m, n)) { bad++; printf("idesc %d %d\n", m, n); }
    }
  printf("mismatches %d\n", bad);
  return bad != 0;
}
'''


def _cutlass_include():
    for root in sys.path:
        for cand in glob.glob(os.path.join(root, "*", "data", "cutlass", "include")) + glob.glob(
                os.path.join(root, "*", "3rdparty", "cutlass", "include")):
            if os.path.exists(os.path.join(cand, "cute", "arch", "mma_sm100_desc.hpp")):
                return cand
    return None


def test_descriptors_match_cutlass_bitfields(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    inc = _cutlass_include()
    if not os.path.exists(nvcc) or inc is None:
        pytest.skip("nvcc or CUTLASS headers not available")
    src = tmp_path / "desc.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "desc"
    r = subprocess.run([nvcc, "-std=c++17", "-I", inc, "-I", REPO, str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    out = subprocess.run([str(exe)], capture_output=True, text=True)
    assert out.returncode == 0 and "mismatches 0" in out.stdout, out.stdout[-2000:]
