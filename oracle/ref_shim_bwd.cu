// ref_shim_bwd.cu -- TEST INFRASTRUCTURE ONLY. Compiles the reference's own
// fp64 backward oracle bwd_ref_f64 (bwd.cu:20-69) and its finite-difference
// loss loss_f64 (bwd.cu:73-105) from the reference source tree (FA_REF_SOURCE)
// and exposes them through C entry points. Both live in an unnamed namespace
// of that file, so they are reached from this same translation unit. The
// driver `main` is renamed; nothing here launches a kernel.
#include <cstdint>
#include <cstring>
#define main fa_reference_bwd_driver_main
#include FA_REF_SOURCE
#undef main

namespace {
std::vector<__half> halves(const uint16_t* p, size_t n) {
  std::vector<__half> out(n);
  std::memcpy(out.data(), p, n * 2);
  return out;
}
}  // namespace

extern "C" void ref_bwd_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                            const uint16_t* dO, double* dq, double* dk, double* dv, int BH, int N,
                            int d, int causal) {
  const size_t n = static_cast<size_t>(BH) * N * d;
  std::vector<double> rq, rk, rv;
  bwd_ref_f64(halves(q, n), halves(k, n), halves(v, n), halves(dO, n), rq, rk, rv, BH, N, d,
              1.0 / std::sqrt(static_cast<double>(d)), causal != 0);
  std::memcpy(dq, rq.data(), n * sizeof(double));
  std::memcpy(dk, rk.data(), n * sizeof(double));
  std::memcpy(dv, rv.data(), n * sizeof(double));
}

extern "C" double ref_loss_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                               const uint16_t* dO, int BH, int N, int d, int causal, int which,
                               size_t idx, double pert) {
  const size_t n = static_cast<size_t>(BH) * N * d;
  return loss_f64(halves(q, n), halves(k, n), halves(v, n), halves(dO, n), BH, N, d,
                  1.0 / std::sqrt(static_cast<double>(d)), causal != 0, which, idx, pert);
}
