// Batched Newton-Schulz orthogonalisation for Muon.
//
// X: (B, m, n) with m <= n, already Frobenius-normalised, bf16.  Each step:
//   A = X X^T            (B, m, m)   symmetric Gram of the short side
//   P = b A + c A A      (B, m, m)
//   X = a X + P X        (B, m, n)
// This version issues the three products as batched tensor-core GEMMs; the
// elementwise combinations are folded into their alpha/beta terms.
#include "../common.cuh"

namespace lrb {

at::Tensor newton_schulz(const at::Tensor& X0, int64_t steps, double a, double b, double c) {
  LRB_CHECK(X0.is_cuda() && X0.dim() == 3 && X0.size(1) <= X0.size(2), "newton_schulz: (B, m, n) with m <= n");
  c10::cuda::CUDAGuard g(X0.device());
  at::Tensor X = X0.contiguous();
  for (int64_t i = 0; i < steps; ++i) {
    at::Tensor A = at::bmm(X, X.transpose(1, 2));
    at::Tensor P = at::baddbmm(A, A, A, /*beta=*/b, /*alpha=*/c);
    X = at::baddbmm(X, P, X, /*beta=*/a, /*alpha=*/1.0);
  }
  return X;
}

}  // namespace lrb
