"""A C++ host program drives the C ABI directly (no Python, no PyTorch on the
path): it reads seeded inputs from files, calls ssm_fwd / ssm_bwd on cudaMalloc
buffers and writes the results back; they must match the NumPy oracle."""

import os
import subprocess

import numpy as np
import pytest

from oracle import selectssm_oracle as O

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "selectssm_b200")

HOST = r'''
#include <cstdio>
#include <cstdlib>
#include <vector>
#include <cuda_runtime.h>
#include "selectssm_b200.h"

static std::vector<float> rd(const char* dir, const char* name, size_t n) {
  std::vector<float> v(n);
  char path[1024];
  snprintf(path, sizeof(path), "%s/%s.bin", dir, name);
  FILE* f = fopen(path, "rb");
  if (!f || fread(v.data(), 4, n, f) != n) { fprintf(stderr, "read %s\n", path); exit(2); }
  fclose(f);
  return v;
}
static float* up(const std::vector<float>& h) {
  float* d; cudaMalloc(&d, h.size() * 4); cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice); return d;
}
static float* zeros(size_t n) { float* d; cudaMalloc(&d, n * 4); cudaMemset(d, 0, n * 4); return d; }
static void wr(const char* dir, const char* name, const float* d, size_t n) {
  std::vector<float> h(n);
  cudaMemcpy(h.data(), d, n * 4, cudaMemcpyDeviceToHost);
  char path[1024];
  snprintf(path, sizeof(path), "%s/%s.out", dir, name);
  FILE* f = fopen(path, "wb"); fwrite(h.data(), 4, n, f); fclose(f);
}

int main(int argc, char** argv) {
  const char* dir = argv[1];
  const int B = atoi(argv[2]), L = atoi(argv[3]), D = atoi(argv[4]), N = 16;
  const size_t act = (size_t)B * L * D, bc = (size_t)B * L * N;
  ssm_params_t p = {};
  p.batch = B; p.seqlen = L; p.dim = D; p.dstate = N;
  p.dtype = SSM_F32; p.bc_dtype = SSM_F32;
  p.flags = SSM_DELTA_SOFTPLUS; p.gate_act = SSM_ACT_SILU;
  p.u = up(rd(dir, "u", act)); p.delta = up(rd(dir, "delta", act)); p.z = up(rd(dir, "z", act));
  p.A = up(rd(dir, "A", (size_t)D * N)); p.Bm = up(rd(dir, "B", bc)); p.Cm = up(rd(dir, "C", bc));
  p.D = up(rd(dir, "D", D)); p.delta_bias = up(rd(dir, "bias", D));
  p.dout = up(rd(dir, "dout", act));
  float* out = zeros(act); p.out = out;
  p.states = zeros(ssm_states_elems(&p));
  float *du = zeros(act), *dd = zeros(act), *dz = zeros(act), *dA = zeros((size_t)D * N), *dB = zeros(bc),
        *dC = zeros(bc), *dD = zeros(D), *db = zeros(D);
  p.du = du; p.ddelta = dd; p.dz = dz; p.dA = dA; p.dB = dB; p.dC = dC; p.dD = dD; p.ddelta_bias = db;
  p.workspace_bytes = ssm_workspace_bytes(&p);
  cudaMalloc(&p.workspace, p.workspace_bytes);
  int st = ssm_fwd(&p, 0);
  if (st == SSM_OK) st = ssm_bwd(&p, 0);
  cudaDeviceSynchronize();
  if (st != SSM_OK) { fprintf(stderr, "status %d: %s [%s]\n", st, ssm_strerror(st), ssm_last_error()); return 1; }
  wr(dir, "out", out, act); wr(dir, "du", du, act); wr(dir, "ddelta", dd, act); wr(dir, "dz", dz, act);
  wr(dir, "dA", dA, (size_t)D * N); wr(dir, "dB", dB, bc); wr(dir, "dC", dC, bc); wr(dir, "dD", dD, D);
  wr(dir, "ddelta_bias", db, D);
  printf("%s ok\n", ssm_version());
  return 0;
}
'''


def test_c_host_program_through_the_abi(tmp_path):
    Bsz, L, D = 2, 300, 64
    inp = O.make_scan_inputs(Bsz, L, D, 16, seed=5)
    inp["bias"] = np.random.default_rng(5).uniform(-0.5, 0.5, D)
    for k, v in inp.items():
        np.ascontiguousarray(v, dtype=np.float32).tofile(tmp_path / f"{k}.bin")
    f32 = {k: np.asarray(v, dtype=np.float32).astype(np.float64) for k, v in inp.items()}
    src = tmp_path / "host.cu"
    src.write_text(HOST)
    exe = tmp_path / "host"
    subprocess.run(["nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O2",
                    "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                    f"-L{PKG}", "-lselectssm_b200", f"-Xlinker=-rpath,{PKG}"], check=True)
    run = subprocess.run([str(exe), str(tmp_path), str(Bsz), str(L), str(D)], capture_output=True, text=True)
    assert run.returncode == 0, run.stderr
    kw = dict(D=f32["D"], z=f32["z"], delta_bias=f32["bias"], delta_softplus=True)
    ref_out = O.selective_scan_fwd(f32["u"], f32["delta"], f32["A"], f32["B"], f32["C"], **kw)
    ref = O.selective_scan_bwd(f32["u"], f32["delta"], f32["A"], f32["B"], f32["C"], f32["dout"], **kw)
    ref["out"] = ref_out
    for name in ("out", "du", "ddelta", "dz", "dA", "dB", "dC", "dD", "ddelta_bias"):
        got = np.fromfile(tmp_path / f"{name}.out", dtype=np.float32).reshape(ref[name].shape)
        assert np.abs(got - ref[name]).max() / np.abs(ref[name]).max() < 1e-4, name
