// ref_shim_fwd.cu -- TEST INFRASTRUCTURE ONLY. Compiles the reference's own
// fp64 forward oracle, attention_ref_f64 (attention.cu:72-102), straight from
// the reference source tree (path given as FA_REF_SOURCE by oracle/Makefile)
// and exposes it through a C entry point. The reference's driver `main` is
// renamed so only the host function is reachable; nothing here launches a
// kernel. Inputs are fp16 bit patterns, layout (BH, N, d), no GQA.
#include <cstdint>
#include <cstring>
#define main fa_reference_attention_driver_main
#include FA_REF_SOURCE
#undef main

extern "C" void ref_attention_f64(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                  double* o, int BH, int N, int d, int causal) {
  const size_t n = static_cast<size_t>(BH) * N * d;
  std::vector<__half> Q(n), K(n), V(n);
  std::memcpy(Q.data(), q, n * 2);
  std::memcpy(K.data(), k, n * 2);
  std::memcpy(V.data(), v, n * 2);
  std::vector<double> O;
  attention_ref_f64(Q, K, V, O, BH, N, d, 1.0 / std::sqrt(static_cast<double>(d)), causal != 0);
  std::memcpy(o, O.data(), n * sizeof(double));
}
