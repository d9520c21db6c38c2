/*
 * CPU oracle for the momentum selective scan and the LinOSS 2x2 scan.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: the parity tests, the
 * smoke check and the CPU-baseline leg of the benchmark call it; the product
 * path (momentummamba_b200) never links or calls it.
 *
 * It is a plain sequential restatement of the reference's recurrences, with
 * OpenMP across independent chains.  Every routine exists twice, once with
 * `double` state (the arbiter the CUDA kernels are compared against) and once
 * with `float` state (the reference's own fp32 arithmetic, used as the timed
 * CPU baseline).  The suffix _f64 / _f32 names the variant.
 *
 * Reference algorithms restated here (paths inside the reference project):
 *   - discretisation  exp(dA), dB*x*alpha       mamba_momentum.py:291-296
 *   - recurrence v = b*v + u ; h = a*h + v       mamba_momentum.py:415-435
 *   - output y = C.h + D*x                       mamba_momentum.py:313-321
 *   - SiLU(z) gate of the block                  mamba_momentum.py:227-229
 *   - softplus(delta + bias) of ssm_momentum     mamba_momentum.py:244-247
 *   - row scan fwd/bwd (momentum_scan_cuda)      momentum_scan_cuda.py:22-87
 *   - PScan fwd/bwd (beta = 0 case of the rows)  pscan.py:160-232
 *   - 2x2 scan x_t = M_t x_{t-1} + F_t           mamba_linoss.py:336-415, :561-605
 *                                                LinOSS_pytorch.py:53-132
 * The gradients are the exact adjoints of those recurrences.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

typedef int64_t i64;

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

#define REAL double
#define SFX(name) name##_f64
#define EXP exp
#define LOG1P log1p
#include "scan_oracle_impl.h"
#undef REAL
#undef SFX
#undef EXP
#undef LOG1P

#define REAL float
#define SFX(name) name##_f32
#define EXP expf
#define LOG1P log1pf
#include "scan_oracle_impl.h"
#undef REAL
#undef SFX
#undef EXP
#undef LOG1P
