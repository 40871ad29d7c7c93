/* gemm_tc.cuh -- interface of the emulated-GEMM kernel (gemm_tc.cu). */
#pragma once

#include "common.cuh"

namespace mpk {

/* The cross products of one call, in accumulation order: plane ia[t] of A
 * times plane ib[t] of B. */
struct GemmTerms {
    int n;
    int ia[16];
    int ib[16];
};

struct GemmArgs {
    const CUtensorMap* tmA;   /* 3D: (contiguous dim, other dim, plane) */
    const CUtensorMap* tmB;
    int m, n, k;
    bool a_mn, b_mn;          /* MN-major operand (op = N for A, op = T for B) */
    bool bf16;                /* operand format: BF16 (true) or FP16 */
    GemmTerms terms;
    float alpha, beta;
    int init_mode;            /* 1 (alpha a power of two, beta 0 or 1): the sum starts at beta*C/alpha */
    float* C;
    long long ldc;
    int* status;
    int num_sms;
};

int gemm_tile_m();
int gemm_tile_n(float beta, int init_mode);   /* B tile width (the K-major box) for a call */
int gemm_tile_k();
cudaError_t launch_gemm_tc(const GemmArgs& g, cudaStream_t s);

}  /* namespace mpk */
