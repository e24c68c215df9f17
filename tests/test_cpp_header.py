"""The reference's C++ declaration, ``hpc_ops_hopper::hopper_gmm_forward``
(reference csrc/hopper_gmm_forward.h:23-25), as a C++ caller written against
that header would use it: include ``include/hopper_gmm_forward.h``, link
``gmm_b200/_C.so``, call with the default ``transb``.

The CPU test compiles such a caller and checks that a host-resident A raises
the reference's message (reference csrc/hopper_gmm_forward.cu:375); the GPU
test runs a real call and a bad ``batch_sizes`` through the same caller.
"""

import os
import subprocess

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
TORCH_DIR = os.path.dirname(torch.__file__)
LIB = os.path.join(ROOT, "gmm_b200", "_C.so")

CPU_CALLER = r"""
#include <ATen/ATen.h>
#include <iostream>
#include "hopper_gmm_forward.h"
int main() {
  at::Tensor A = at::zeros({10, 64}, at::kBFloat16);
  at::Tensor B = at::zeros({2, 64, 32}, at::kBFloat16);
  at::Tensor bs = at::empty({2}, at::kLong);
  bs[0] = 4;
  bs[1] = 6;
  try {
    hpc_ops_hopper::hopper_gmm_forward(A, B, bs);  // transb defaults to false
    std::cout << "no error\n";
    return 1;
  } catch (const c10::Error& e) {
    std::cout << e.what_without_backtrace() << "\n";
    return 0;
  }
}
"""

GPU_CALLER = r"""
#include <ATen/ATen.h>
#include <iostream>
#include "hopper_gmm_forward.h"
int main() {
  auto opt = at::TensorOptions().dtype(at::kBFloat16).device(at::kCUDA, 0);
  at::manual_seed(7);
  at::Tensor A = at::randn({300, 64}, opt);
  at::Tensor B = at::randn({3, 64, 96}, opt);
  at::Tensor bs = at::empty({3}, at::kLong);
  bs[0] = 100; bs[1] = 0; bs[2] = 200;
  at::Tensor D = hpc_ops_hopper::hopper_gmm_forward(A, B, bs);
  at::Tensor want0 = at::matmul(A.narrow(0, 0, 100).to(at::kFloat), B[0].to(at::kFloat));
  at::Tensor want2 = at::matmul(A.narrow(0, 100, 200).to(at::kFloat), B[2].to(at::kFloat));
  const double e0 = (D.narrow(0, 0, 100).to(at::kFloat) - want0).abs().max().item<double>();
  const double e2 = (D.narrow(0, 100, 200).to(at::kFloat) - want2).abs().max().item<double>();
  std::cout << "max_err " << std::max(e0, e2) << " scale " << want2.abs().max().item<double>() << "\n";
  bs[2] = 199;
  try {
    hpc_ops_hopper::hopper_gmm_forward(A, B, bs, false);
    std::cout << "no error\n";
    return 1;
  } catch (const c10::Error& e) {
    std::cout << e.what_without_backtrace() << "\n";
  }
  return 0;
}
"""


def _build(tmp_path, src, cuda):
    if not os.path.exists(LIB):
        pytest.skip("gmm_b200/_C.so is not built")
    cpp = tmp_path / "caller.cpp"
    cpp.write_text(src)
    exe = tmp_path / "caller"
    libs = ["-lc10", "-ltorch_cpu"] + (["-lc10_cuda", "-ltorch_cuda", "-ltorch"] if cuda else [])
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-std=c++17", "-O0", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-I", os.path.join(TORCH_DIR, "include"), "-I", os.path.join(ROOT, "include"),
           str(cpp), "-o", str(exe),
           "-L", os.path.join(ROOT, "gmm_b200"), "-l:_C.so", f"-Wl,-rpath,{os.path.join(ROOT, 'gmm_b200')}",
           "-L", os.path.join(TORCH_DIR, "lib"), f"-Wl,-rpath,{os.path.join(TORCH_DIR, 'lib')}",
           "-Wl,--no-as-needed", *libs]
    subprocess.run(cmd, check=True, capture_output=True, text=True, timeout=600)
    return exe


def test_cpp_caller_links_and_gets_reference_messages(tmp_path):
    exe = _build(tmp_path, CPU_CALLER, cuda=False)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "A must be a contiguous CUDA tensor" in r.stdout


@pytest.mark.gpu
def test_cpp_caller_on_gpu(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    exe = _build(tmp_path, GPU_CALLER, cuda=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.splitlines()
    err, scale = float(lines[0].split()[1]), float(lines[0].split()[3])
    assert err <= 1.6e-2 * (1.0 + scale), lines[0]  # bf16 tolerance, rtol = atol
    assert "Sum of batch_sizes (299) must equal A.size(0) (300)" in r.stdout
