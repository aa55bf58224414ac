# Compiles the reference's own host harnesses -- validators and loadtests for the
# elementwise / reduction path and the Q8 GEMVs -- from their sources where they lie in the
# reference tree, into oracle/_ref/ (git-ignored; the binaries travel to the GPU
# box with the snapshot).  Nothing is copied out of the reference tree.
#
# Include set and flags follow the reference Makefile (Makefile:6-9, :60, :67-68);
# v_rmsnorm_validate is built at -O0 as the reference builds it (Makefile:60).
# The reference's engine itself is NASM and cannot be assembled here (no nasm).
# The reference tree: REF=... on the command line, else $V7_REFERENCE_DIR, else
# a `reference` checkout beside this repository (this file runs from oracle/).
REF ?= $(or $(V7_REFERENCE_DIR),$(abspath ../../reference))
OUT := _ref
CXX ?= g++
CPPFLAGS_REF := -D_GNU_SOURCE -I$(REF)/src/linux/compat -I$(REF)/src/linux -I$(REF)/src -I$(REF)/tools -I$(REF)/tools/zydis_stub
CXXFLAGS_REF := -O2 -std=c++17 -w
LIBS_REF := -ldl -lm -pthread

VALIDATORS := v_rmsnorm_validate v_add_inplace_validate v_quantize_validate v_swiglu_validate v_matmul_validate
LOADTESTS := b_rmsnorm_loadtest b_fused_add_rmsnorm_loadtest b_rmsnorm_rope_loadtest b_add_inplace_loadtest \
	b_swiglu_q8_loadtest b_swiglu_loadtest
BINS := $(addprefix $(OUT)/,$(VALIDATORS) $(LOADTESTS))

.PHONY: all
all: $(BINS)

$(OUT):
	mkdir -p $@

$(OUT)/v_rmsnorm_validate: $(REF)/tools/v_rmsnorm_validate.cpp | $(OUT)
	$(CXX) $(CPPFLAGS_REF) $(CXXFLAGS_REF) -O0 $< -o $@ $(LIBS_REF)

$(OUT)/%: $(REF)/tools/%.cpp | $(OUT)
	$(CXX) $(CPPFLAGS_REF) $(CXXFLAGS_REF) $< -o $@ $(LIBS_REF)
