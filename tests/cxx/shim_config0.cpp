// A C++ host binding libqb_gdn.so as quotebound's own deltanet code would: the gated_delta /
// gated_delta_vjp shim of INTEGRATION.md over include/qb_gdn.h, exceptions on the C++ side as
// src/delta_grad.cpp:164-170 throws them.  Test driver for tests/test_cxx_shim.py:
//   shim_config0 <inputs.bin> <outputs.bin>
// inputs.bin: int32 B, T, Hk, Hv, Dk, Dv, then float32 q, k, v, g, beta, state, dy, dstate (float32
// activations); outputs.bin: float32 y, state_out, dq, dk, dv, dg, dbeta, dstate0.
#include <cuda_runtime.h>

#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

#include "qb_gdn.h"

static void check(int rc, const char* err) {
  if (rc) throw std::runtime_error(err);
}

// ---- the shim -----------------------------------------------------------------------
void gated_delta(const qb_gdn_desc& d, const void* q, const void* k, const void* v, const float* g,
                 const float* beta, const float* state, void* y, float* state_out, void* saved, void* ws,
                 int64_t ws_bytes, cudaStream_t stream) {
  char err[512];
  check(qb_gdn_fwd(&d, q, k, v, g, beta, state, y, state_out, saved, ws, ws_bytes, stream, err, sizeof err), err);
}

void gated_delta_vjp(const qb_gdn_desc& d, const void* q, const void* k, const void* v, const float* g,
                     const float* beta, const float* state, const void* dy, const float* dstate, const void* saved,
                     void* dq, void* dk, void* dv, float* dg, float* dbeta, float* dstate0, void* ws,
                     int64_t ws_bytes, cudaStream_t stream) {
  char err[512];
  check(qb_gdn_bwd(&d, q, k, v, g, beta, state, dy, dstate, saved, dq, dk, dv, dg, dbeta, dstate0, ws, ws_bytes,
                   stream, err, sizeof err),
        err);
}

// ---- driver ---------------------------------------------------------------------------------------
static void cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

struct Dev {
  void* p = nullptr;
  size_t n = 0;
  explicit Dev(size_t bytes) : n(bytes) { cuda(cudaMalloc(&p, bytes ? bytes : 1), "cudaMalloc"); }
  ~Dev() { cudaFree(p); }
  float* f() const { return static_cast<float*>(p); }
};

int main(int argc, char** argv) {
  try {
    if (argc != 3) throw std::runtime_error("usage: shim_config0 inputs.bin outputs.bin");
    FILE* in = std::fopen(argv[1], "rb");
    if (!in) throw std::runtime_error("cannot open inputs");
    int32_t s[6];
    if (std::fread(s, 4, 6, in) != 6) throw std::runtime_error("short header");
    const int B = s[0], T = s[1], Hk = s[2], Hv = s[3], Dk = s[4], Dv = s[5];
    const size_t nq = (size_t)B * T * Hk * Dk, nv = (size_t)B * T * Hv * Dv, ng = (size_t)B * T * Hv,
                 ns = (size_t)B * Hv * Dv * Dk;
    const size_t sizes[8] = {nq, nq, nv, ng, ng, ns, nv, ns};
    std::vector<Dev*> x;
    for (size_t n : sizes) {
      std::vector<float> h(n);
      if (std::fread(h.data(), 4, n, in) != n) throw std::runtime_error("short inputs");
      x.push_back(new Dev(n * 4));
      cuda(cudaMemcpy(x.back()->p, h.data(), n * 4, cudaMemcpyHostToDevice), "upload");
    }
    std::fclose(in);

    qb_gdn_desc d{};
    d.B = B, d.T = T, d.Hk = Hk, d.Hv = Hv, d.Dk = Dk, d.Dv = Dv;
    d.in_dtype = d.out_dtype = QB_DTYPE_F32;
    d.algo = QB_ALGO_AUTO;
    char err[512];
    const int64_t wf = qb_gdn_workspace_bytes(&d, QB_OP_FWD, err, sizeof err);
    const int64_t wb = qb_gdn_workspace_bytes(&d, QB_OP_BWD, err, sizeof err);
    const int64_t sv = qb_gdn_saved_bytes(&d, err, sizeof err);
    if (wf < 0 || wb < 0 || sv < 0) throw std::runtime_error(err);
    Dev ws_f(wf), ws_b(wb), saved(sv);
    const size_t on[8] = {nv, ns, nq, nq, nv, ng, ng, ns};
    std::vector<Dev*> o;
    for (size_t n : on) o.push_back(new Dev(n * 4));
    cudaStream_t st;
    cuda(cudaStreamCreate(&st), "stream");
    // training forward (the chunk-start states kept), then the VJP from them
    gated_delta(d, x[0]->p, x[1]->p, x[2]->p, x[3]->f(), x[4]->f(), x[5]->f(), o[0]->p, o[1]->f(), saved.p, ws_f.p, wf,
                st);
    gated_delta_vjp(d, x[0]->p, x[1]->p, x[2]->p, x[3]->f(), x[4]->f(), x[5]->f(), x[6]->p, x[7]->f(), saved.p,
                    o[2]->p, o[3]->p, o[4]->p, o[5]->f(), o[6]->f(), o[7]->f(), ws_b.p, wb, st);
    int32_t code = -1;
    check(qb_gdn_status(ws_b.p, &code, st, err, sizeof err), err);
    if (code) throw std::runtime_error("device status " + std::to_string(code));
    // a bad shape must come back as an error, not a crash
    qb_gdn_desc bad = d;
    bad.Hv = 3;
    bool threw = false;
    try {
      gated_delta(bad, x[0]->p, x[1]->p, x[2]->p, x[3]->f(), x[4]->f(), x[5]->f(), o[0]->p, o[1]->f(), nullptr,
                  ws_f.p, wf, st);
    } catch (const std::runtime_error& e) {
      threw = std::string(e.what()).find("multiple of key heads") != std::string::npos;
    }
    if (!threw) throw std::runtime_error("a bad shape was not rejected");
    cuda(cudaStreamSynchronize(st), "sync");
    FILE* out = std::fopen(argv[2], "wb");
    if (!out) throw std::runtime_error("cannot open outputs");
    for (size_t i = 0; i < o.size(); ++i) {
      std::vector<float> h(on[i]);
      cuda(cudaMemcpy(h.data(), o[i]->p, on[i] * 4, cudaMemcpyDeviceToHost), "download");
      std::fwrite(h.data(), 4, on[i], out);
    }
    std::fclose(out);
    for (Dev* p : x) delete p;
    for (Dev* p : o) delete p;
    cudaStreamDestroy(st);
    std::printf("shim ok: %s\n", qb_gdn_version());
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "shim_config0: %s\n", e.what());
    return 1;
  }
}
