# Builds the REFERENCE's own CPU KernelModule executor from its sources, in
# place, into oracle/_ref/ (git-ignored; the built files travel to the GPU box).
#
# Test infrastructure only: the products are the parity checker and the timed
# CPU baseline (`cpu_baseline.kind = "reference"`), never part of the shipped path.
#
# The reference's CMake build needs -std=c++26, which GCC 13 rejects, so this
# recipe compiles every library translation unit directly with -std=c++23
# (the sources use nothing newer). Nothing is copied out of the reference tree:
# objects are written under oracle/_ref/obj/.
#
#   make -f oracle/ref.mk REF=/path/to/reference -j8
ifeq ($(strip $(REF)),)
$(error REF=<reference source tree> is required)
endif
OUT      ?= oracle/_ref
CXX      ?= g++
CXXFLAGS ?= -std=c++23 -O2 -fPIC -fno-exceptions -fno-rtti -w -pthread

INCS := $(foreach d,compiler runtime backends/cpu polyhedral autotuner superopt fastkernel,-I$(REF)/$(d)/include)
SRCS := $(shell find $(REF)/compiler/src $(REF)/runtime/src $(REF)/backends/cpu/src \
          $(REF)/polyhedral/src $(REF)/autotuner/src $(REF)/superopt/src \
          $(REF)/fastkernel/src -name '*.cpp' 2>/dev/null | sort)
OBJS := $(patsubst $(REF)/%.cpp,$(OUT)/obj/%.o,$(SRCS))

all: $(OUT)/libmlkref.so $(OUT)/ref_loader_check

$(OUT)/obj/%.o: $(REF)/%.cpp
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) $(INCS) -c $< -o $@

$(OUT)/libmlkref_core.a: $(OBJS)
	@rm -f $@
	ar rcs $@ $^

# C-ABI driver over executeKernelOnBuffers (our code, reference headers).
$(OUT)/libmlkref.so: oracle/ref_driver.cpp oracle/ref_modules.h $(OUT)/libmlkref_core.a
	$(CXX) $(CXXFLAGS) $(INCS) -shared oracle/ref_driver.cpp \
	  -Wl,--whole-archive $(OUT)/libmlkref_core.a -Wl,--no-whole-archive \
	  -ldl -o $@

# Drop-in check: the reference's own loadKernelLibrary + LoadedKernel::run
# driving our mlk_kernel shim.
$(OUT)/ref_loader_check: oracle/ref_loader_check.cpp oracle/ref_modules.h $(OUT)/libmlkref_core.a
	$(CXX) $(CXXFLAGS) $(INCS) oracle/ref_loader_check.cpp \
	  $(OUT)/libmlkref_core.a -ldl -o $@

.PHONY: all
