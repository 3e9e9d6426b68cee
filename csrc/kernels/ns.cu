// Batched Newton-Schulz orthogonalisation for Muon.
//
// X: (B, m, n) with m <= n, already Frobenius-normalised, bf16.  Each step:
//   A = X X^T            (B, m, m)   symmetric Gram of the short side
//   P = c A A + b A      (B, m, m)   (A A = A A^T: the K-major operand is A itself)
//   X = P X + a X        (B, m, n)   (X read MN-major: no transposed copy)
// The three products run on the batched tcgen05 GEMM (gemm_batched_sm100.cu)
// with the elementwise combinations folded into its axpby epilogue, so one
// iteration is three launches and X ping-pongs between two buffers.
#include "../common.cuh"

namespace lrb {

void gemm_batched(const at::Tensor& A, const at::Tensor& B, bool b_mn, const at::Tensor& C,
                  const c10::optional<at::Tensor>& D, double alpha, double beta);

at::Tensor newton_schulz(const at::Tensor& X0, int64_t steps, double a, double b, double c) {
  LRB_CHECK(X0.is_cuda() && X0.dim() == 3 && X0.size(1) <= X0.size(2), "newton_schulz: (B, m, n) with m <= n");
  c10::cuda::CUDAGuard g(X0.device());
  const int64_t Bt = X0.size(0), m = X0.size(1), n = X0.size(2);
  const bool native_ok = X0.scalar_type() == at::kBFloat16 && m % 8 == 0 && n % 8 == 0;
  if (!native_ok) {  // fp16 / fp32 or rows that TMA cannot address: library batched GEMMs
    at::Tensor X = X0.contiguous();
    for (int64_t i = 0; i < steps; ++i) {
      at::Tensor A = at::bmm(X, X.transpose(1, 2));
      at::Tensor P = at::baddbmm(A, A, A, /*beta=*/b, /*alpha=*/c);
      X = at::baddbmm(X, P, X, /*beta=*/a, /*alpha=*/1.0);
    }
    return X;
  }
  at::Tensor X = X0.contiguous();  // read only: the iterates alternate between two new buffers
  at::Tensor bufs[2] = {at::empty_like(X), steps > 1 ? at::empty_like(X) : at::Tensor()};
  at::Tensor A = at::empty({Bt, m, m}, X.options());
  at::Tensor P = at::empty({Bt, m, m}, X.options());
  for (int64_t i = 0; i < steps; ++i) {
    at::Tensor& out = bufs[i % 2];
    gemm_batched(X, X, false, A, c10::nullopt, 1.0, 0.0);  // A = X X^T
    gemm_batched(A, A, false, P, A, c, b);                  // P = c A A + b A
    gemm_batched(P, X, true, out, X, 1.0, a);               // X' = P X + a X
    X = out;
  }
  return X;
}

}  // namespace lrb
