/* Stand-in for MSVC's <intrin.h> so the reference sources compile with g++
 * on Linux: only __cpuid(int regs[4], int leaf) is used
 * (cpp/dequant_k.cpp:114-120).  Test infrastructure only. */
#pragma once
#include <cpuid.h>
#undef __cpuid
static inline void __cpuid(int regs[4], int leaf) {
    unsigned a = 0, b = 0, c = 0, d = 0;
    __get_cpuid((unsigned)leaf, &a, &b, &c, &d);
    regs[0] = (int)a; regs[1] = (int)b; regs[2] = (int)c; regs[3] = (int)d;
}
