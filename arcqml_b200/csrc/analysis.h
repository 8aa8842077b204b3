// analysis.h — analysis of device states (analysis.cu): probabilities, marginals, Bloch
// vectors, overlaps and the adjoint cotangents of those outputs.
#pragma once

#include <vector>

#include "rt_internal.h"

namespace arcqml {

// A validated qubit selection of an n-qubit state: display order disp (descending qubits, the
// first the most significant bit of a marginal's output index), the same qubits ascending, and
// whether every qubit is selected (then a basis index is its own bin).
struct Selection {
    uint32_t k;
    int32_t identity;
    uint8_t disp[64];
    uint8_t asc[64];
};
Selection make_selection(uint32_t n, const std::vector<uint32_t> &qubits);

// out[row][i] = |psi_row[i]|^2 (device).
void probabilities_device(const double2 *a, size_t batch, uint32_t n, double *out, cudaStream_t s);
// out[row][m] = sum of |psi_row[i]|^2 over the basis indices i of bin m (device, 2^k per row).
void marginal_device(const double2 *a, size_t batch, uint32_t n, const Selection &S,
                     double *out, ThreadContext &ctx, cudaStream_t s);
// xyz[3 row + c] = <X_q>, <Y_q>, <Z_q> of each row (host).
void bloch_device(const double2 *a, size_t batch, uint32_t n, uint32_t q, double *xyz,
                  ThreadContext &ctx, cudaStream_t s);
// out[2 row], out[2 row + 1] = real and imaginary part of <lhs_row|rhs_row> (host).
void overlap_device(const double2 *l, const double2 *r, size_t batch, uint32_t n, double *out,
                    ThreadContext &ctx, cudaStream_t s);
// lam[row][i] = g[row][bin(i)] psi_row[i] (g device, 2^k per row).
void probability_cotangent_device(const double2 *psi, size_t batch, uint32_t n,
                                  const Selection &S, const double *g, double2 *lam,
                                  cudaStream_t s);
// out[row] = alpha[row] x[row], alpha complex (host, 2 doubles per row).
void scaled_copy_device(const double2 *x, size_t batch, uint32_t n, const double *alpha_host,
                        double2 *out, ThreadContext &ctx, cudaStream_t s);

}  // namespace arcqml
