/* Linux stand-in for the MSVC <intrin.h> the reference's native sources include.
 *
 * Test infrastructure only: used by oracle/Makefile to compile the reference's
 * CPU kernels into oracle/_ref/ so they can serve as the parity checker and the
 * timed CPU baseline.  Only the cpuid entry points those files call are
 * provided.  GCC's <cpuid.h> already defines __cpuidex(int[4], int, int) as a
 * function, but __cpuid as a 5-argument macro; the MSVC form takes
 * (int[4], leaf), so the macro is replaced by a function of that shape.
 */
#pragma once
#include <cpuid.h>
#include <immintrin.h>

#undef __cpuid
static inline void __cpuid(int regs[4], int leaf) {
    __cpuid_count(leaf, 0, regs[0], regs[1], regs[2], regs[3]);
}
