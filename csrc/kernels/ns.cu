// Batched Newton-Schulz orthogonalisation for Muon.
//
// X: (B, m, n) with m <= n, already Frobenius-normalised, bf16.  Each step:
//   A = X X^T            (B, m, m)   symmetric Gram of the short side
//   P = c A A + b A      (B, m, m)   (A A = A A^T: the K-major operand is A itself)
//   X = P X + a X        (B, m, n)   (X read MN-major: no transposed copy)
// The three products run on the batched CTA-pair tcgen05 GEMM
// (gemm_pair_sm100.cu: 3-D tensor maps over the batch, 256 x 256 tiles per TPC)
// with the elementwise combinations folded into its axpby epilogue (D staged by
// TMA), so one iteration is three launches and X ping-pongs between two
// buffers.  LRB_NS_GEMM=batched selects the one-CTA batched kernel
// (gemm_batched_sm100.cu) instead.
#include "../common.cuh"

#include <cstdlib>
#include <string>

namespace lrb {

void gemm_batched(const at::Tensor& A, const at::Tensor& B, bool b_mn, const at::Tensor& C,
                  const c10::optional<at::Tensor>& D, double alpha, double beta);
void gemm_pair(const at::Tensor& A, const at::Tensor& B, bool a_mn, bool b_mn, at::Tensor& C, bool accumulate,
               double alpha);
void gemm_pair_axpby(const at::Tensor& A, const at::Tensor& B, bool b_mn, at::Tensor& C, const at::Tensor& D,
                     double alpha, double beta);

at::Tensor newton_schulz(const at::Tensor& X0, int64_t steps, double a, double b, double c) {
  LRB_CHECK(X0.is_cuda() && X0.dim() == 3 && X0.size(1) <= X0.size(2), "newton_schulz: (B, m, n) with m <= n");
  c10::cuda::CUDAGuard g(X0.device());
  bind_device(X0.get_device());
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
  static const bool one_cta = [] {
    const char* e = std::getenv("LRB_NS_GEMM");
    return e != nullptr && std::string(e) == "batched";
  }();
  for (int64_t i = 0; i < steps; ++i) {
    at::Tensor& out = bufs[i % 2];
    if (one_cta) {
      gemm_batched(X, X, false, A, c10::nullopt, 1.0, 0.0);  // A = X X^T
      gemm_batched(A, A, false, P, A, c, b);                  // P = c A A + b A
      gemm_batched(P, X, true, out, X, 1.0, a);               // X' = P X + a X
    } else {
      gemm_pair(X, X, false, false, A, false, 1.0);           // A = X X^T
      gemm_pair_axpby(A, A, false, P, A, c, b);               // P = c A A + b A
      gemm_pair_axpby(P, X, true, out, X, 1.0, a);            // X' = P X + a X
    }
    X = out;
  }
  return X;
}

}  // namespace lrb
