# The reference's own runtime, compiled for this x86 host from its unmodified C sources (TEST INFRASTRUCTURE ONLY: the
# parity oracle's pin, and bench.py's reference arm). Output only under oracle/_ref/.
#
#   make -C oracle -f ref.mk REF=<checkout of the reference repository>
#
# The sources include <arm_neon.h>; -Ineon puts our scalar stand-in (neon/arm_neon.h, written from the Arm ARM) in its
# place. The two inline-assembly GEMM K-block headers are skipped by defining their include guards, and our scalar
# restatements (neon/kblock_f32.h, neon/kblock_f16.h) are force-included instead. __fp16 is _Float16 (x86 GCC's IEEE
# half type); -fexcess-precision=16 rounds every scalar half operation to half, as AArch64 does. The dotprod v3.0
# kernels (src/rt_ops_dot.c, src/gemm_s8.c, src/wino.c, src/wino_s0.c) pin AArch64 registers and are left out
# (ref_stubs.c). -O3 lets GCC vectorize the stand-in's lane loops (the same IEEE lane operations, no reassociation);
# src/v24_fe.c is compiled without vectorization, which hits a GCC 13 internal error there.
REF ?=
SRC = $(REF)/src
OUT = _ref
CC ?= gcc
CFLAGS = -O3 -fPIC -std=gnu11 -ffp-contract=off -march=x86-64-v3 -fno-fast-math \
         -fexcess-precision=16 -D__fp16=_Float16 -Ineon -I$(SRC) -DGEMM_F32_KBLOCK_H -DGEMM_F16_KBLOCK_H \
         -include neon/kblock_f32.h -include neon/kblock_f16.h -w
# the reference Makefile's RT_BASE + V24_BASE + RT_A76 + V24_A76 (Makefile:22-27) without the dotprod v3.0 family
NAMES = rt_pkg rt_pool rt_ops_f32 rt_ops_f32x fe_dbimg wino_f32 rt_ops_s8n gemm_s8n proto_s8n pc_kern_f32 gemv \
        v24_model v24_ref v24_api v24_fe bnneon v24_f32 gemm_f32 \
        rt_ops_f16 pc_kern_f16 pc_proto_s8 v24_fast gemm_f16 kern_f16
OBJS = $(patsubst %,$(OUT)/obj/%.o,$(NAMES)) $(OUT)/obj/ref_stubs.o
STANDIN = neon/arm_neon.h neon/kblock_f32.h neon/kblock_f16.h arm_emu.h

$(OUT)/libbnneon_ref.so: $(OBJS)
	$(CC) -shared -o $@ $(OBJS) -Wl,--wrap=getauxval -Wl,--no-undefined -lm -lpthread

$(OUT)/obj/v24_fe.o: CFLAGS += -fno-tree-vectorize
$(OUT)/obj/%.o: $(SRC)/%.c $(STANDIN) ref.mk
	@mkdir -p $(OUT)/obj
	$(CC) $(CFLAGS) -c -o $@ $<

$(OUT)/obj/ref_stubs.o: ref_stubs.c ref.mk
	@mkdir -p $(OUT)/obj
	$(CC) $(CFLAGS) -c -o $@ $<

clean:
	rm -rf $(OUT)
.PHONY: clean
