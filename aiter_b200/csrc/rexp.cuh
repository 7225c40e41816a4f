// exp and sigmoid of the routing arithmetic contract, shared by the routing kernels
// (routing.cu, topk_sigmoid in moe_misc.cu) and restated bit for bit by
// oracle/routing.py (`rexp`, `_sigmoid`).
//
// rexp(x): Cody & Waite's additive range reduction x = n ln2 + r, |r| <= ln2/2,
// with ln 2 split into a head of 21 significant bits (so n * head is exact for the
// |n| <= 160 used here) and a tail; e^r by its degree-13 Taylor polynomial
// (coefficients 1/i! rounded to double, Horner's rule); both in IEEE double with
// separately rounded multiplies and adds (__dmul_rn / __dadd_rn are never contracted
// into FMAs), then times 2^n (exact) and rounded once to fp32.  The truncation error
// is below 2^-57 relative and the double rounding errors a few double ulps, so the
// result is the correctly rounded e^x except when e^x lies within about 2^-50
// relative of an fp32 rounding boundary.
#pragma once

namespace abd {

__device__ __forceinline__ float rexp(float x) {
    if (x != x) return x;
    if (x > 100.0f) return INFINITY;
    if (x < -110.0f) return 0.0f;
    const double kLog2e = 0x1.71547652b82fep+0;
    const double kLn2Hi = 0x1.62e42p-1;
    const double kLn2Lo = 0x1.fdf473de6af28p-22;
    const double d = (double)x;
    const double n = rint(__dmul_rn(d, kLog2e));
    const double r = __dadd_rn(__dadd_rn(d, -__dmul_rn(n, kLn2Hi)), -__dmul_rn(n, kLn2Lo));
    // 1/i! for i = 13 .. 0
    double p = 0x1.6124613a86d09p-33;
    p = __dadd_rn(__dmul_rn(p, r), 0x1.1eed8eff8d898p-29);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.ae64567f544e4p-26);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.27e4fb7789f5cp-22);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.71de3a556c734p-19);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.a01a01a01a01ap-16);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.a01a01a01a01ap-13);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.6c16c16c16c17p-10);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.1111111111111p-7);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.5555555555555p-5);
    p = __dadd_rn(__dmul_rn(p, r), 0x1.5555555555555p-3);
    p = __dadd_rn(__dmul_rn(p, r), 0x1p-1);
    p = __dadd_rn(__dmul_rn(p, r), 1.0);
    p = __dadd_rn(__dmul_rn(p, r), 1.0);
    const double scale = __longlong_as_double((long long)((int)n + 1023) << 52);
    return __double2float_rn(__dmul_rn(p, scale));
}

// sigmoid(x) = 1 / (1 + e^-x), each step rounded to fp32.
__device__ __forceinline__ float rsigmoid(float x) {
    return __frcp_rn(__fadd_rn(1.0f, rexp(-x)));
}

}  // namespace abd
