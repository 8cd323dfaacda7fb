// Host build of crmath.h (same source as the device code) so the CPU test
// suite can check the correctly-rounded log2/exp2 against an independent
// extended-precision evaluation.  Not part of the product path.
#include "crmath.h"

extern "C" {
float crm_log2f(float x) { return crmath::cr_log2f<false>(x); }
float crm_exp2f(float y) { return crmath::cr_exp2f<false>(y); }
float crm_log2f_slow(float x) { return crmath::cr_log2f<true>(x); }
float crm_exp2f_slow(float y) { return crmath::cr_exp2f<true>(y); }
// vector forms for fast sweeps
void crm_log2f_v(const float* x, float* y, long n, int slow) {
    for (long i = 0; i < n; ++i) y[i] = slow ? crmath::cr_log2f<true>(x[i]) : crmath::cr_log2f<false>(x[i]);
}
void crm_exp2f_v(const float* x, float* y, long n, int slow) {
    for (long i = 0; i < n; ++i) y[i] = slow ? crmath::cr_exp2f<true>(x[i]) : crmath::cr_exp2f<false>(x[i]);
}
}
extern "C" void crm_pow4_v(const float* x, float p, float* y, long n) {
    for (long i = 0; i + 4 <= n; i += 4) {
        float a[4] = {x[i], x[i + 1], x[i + 2], x[i + 3]}, o[4];
        crmath::cr_pow2log2<4>(a, p, o);
        for (int j = 0; j < 4; ++j) y[i + j] = o[j];
    }
}
