/* Glue for the x86 build of the reference's own sources (TEST INFRASTRUCTURE ONLY; built by oracle/ref.mk into
 * oracle/_ref/, loaded only by tests/ and bench.py's reference arm).
 *
 * 1. The dotprod kernel family of BirdNET v3.0 packages (src/rt_ops_dot.c over src/gemm_s8.c and src/wino_s0.c) pins
 *    AArch64 registers in its inline assembly and cannot be compiled for x86: its registry table is empty here, so a
 *    package that needs those opcodes is refused by the reference's own loader ("no kernel"). No v2.4 or Perch package
 *    uses them.
 * 2. The reference picks a package path by the CPU's AArch64 HWCAP bits (src/bnneon.c:39-45). The x86 build runs the
 *    NEON intrinsics through the scalar stand-in (oracle/neon/arm_neon.h), which implements the fp16 arithmetic and
 *    SDOT instructions those paths need, so getauxval(AT_HWCAP) answers with asimdhp and asimddp set (the build links
 *    with --wrap=getauxval). */
#include <stdint.h>
#include <sys/auxv.h>

#include "rt.h"
#include "rt_ops.h"

const rt_kernel rt_k_dot[RT_OP_N];

unsigned long __real_getauxval(unsigned long type);
unsigned long __wrap_getauxval(unsigned long type) {
  if (type == AT_HWCAP) return (1ul << 10) | (1ul << 20); /* HWCAP_ASIMDHP | HWCAP_ASIMDDP (arm64 uapi hwcap.h) */
  return __real_getauxval(type);
}
