/*
 * CPU restatement of the reference selective-scan math -- TEST INFRASTRUCTURE ONLY.
 * Instantiates scan_ref_impl.h in double (parity oracle, *_f64) and float (timed CPU
 * baseline, *_f32).  Built by oracle/build.py into oracle/_build/libscan_ref.so.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define REAL double
#define SUFFIX f64
#define EXP exp
#define LOG1P log1p
#include "scan_ref_impl.h"
#undef REAL
#undef SUFFIX
#undef EXP
#undef LOG1P

#define REAL float
#define SUFFIX f32
#define EXP expf
#define LOG1P log1pf
#include "scan_ref_impl.h"
#undef REAL
#undef SUFFIX
#undef EXP
#undef LOG1P

int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* Threads for the following parallel regions of the calling thread (n > 0).  A launcher
   may have set OMP_NUM_THREADS=1 for its ranks; a host baseline sets its own count. */
void oracle_set_num_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}
