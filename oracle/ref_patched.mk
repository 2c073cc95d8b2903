# Builds a PATCHED copy of the reference: the reference-side changes a
# maintainer would make to plug libmlkb200 in (oracle/ref_patches/*.patch),
# applied to a copy of the reference sources under oracle/_ref/patched/src
# (git-ignored; the reference tree itself is never written), compiled and
# linked with our integration check. Test infrastructure only.
#
#   make -f oracle/ref_patched.mk REF=<reference source tree> -j8
#
# The patches:
#   01-backend-driver   accept sm_<digits>a/f arch names; load a prebuilt GPU
#                       library that learns the module via mlk_bind_module;
#                       read mlk_last_status after a legacy-form call
#   02-fastkernel       the NativeCuda search path on a prebuilt library
#                       (Tier1 modules), and a declared ULP-bounded identity
#                       policy for Cuda candidates
#   03-multi-output-lowering  each output's Store / Call targets its own buffer
#   04-poly-bench-b200  `mlk-poly bench --b200-lib=L`: a b200 row per case and
#                       a suite at BASELINE shapes (built here as mlk-poly)
ifeq ($(strip $(REF)),)
$(error REF=<reference source tree> is required)
endif
OUT      := oracle/_ref/patched
SRC      := $(OUT)/src
CXX      ?= g++
CXXFLAGS ?= -std=c++23 -O2 -fPIC -fno-exceptions -fno-rtti -w -pthread
PATCHES  := $(sort $(wildcard oracle/ref_patches/*.patch))
DIRS     := compiler runtime backends polyhedral autotuner superopt fastkernel tools

all: $(SRC)/.applied
	@$(MAKE) --no-print-directory -f oracle/ref_patched.mk REF=$(REF) build

# Fresh copy + patches whenever a patch changes.
$(SRC)/.applied: $(PATCHES)
	rm -rf $(SRC)
	mkdir -p $(SRC)
	cd $(REF) && cp -r $(DIRS) $(abspath $(SRC))/
	set -e; for p in $(PATCHES); do patch -s -d $(SRC) -p1 < $$p; done
	touch $@

ifneq ($(wildcard $(SRC)/.applied),)
INCS := $(foreach d,compiler runtime backends/cpu polyhedral autotuner superopt fastkernel,-I$(SRC)/$(d)/include)
SRCS := $(shell find $(SRC)/compiler/src $(SRC)/runtime/src $(SRC)/backends/cpu/src \
          $(SRC)/polyhedral/src $(SRC)/autotuner/src $(SRC)/superopt/src \
          $(SRC)/fastkernel/src -name '*.cpp' | sort)
OBJS := $(patsubst $(SRC)/%.cpp,$(OUT)/obj/%.o,$(SRCS))

$(OUT)/obj/%.o: $(SRC)/%.cpp $(SRC)/.applied
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) $(INCS) -c $< -o $@

$(OUT)/libmlkref_patched.a: $(OBJS)
	@rm -f $@
	ar rcs $@ $^

$(OUT)/ref_integration_check: oracle/ref_integration_check.cpp oracle/ref_modules.h $(OUT)/libmlkref_patched.a
	$(CXX) $(CXXFLAGS) $(INCS) oracle/ref_integration_check.cpp $(OUT)/libmlkref_patched.a \
	  -ldl -o $@

POLY := $(wildcard $(SRC)/tools/mlk-poly/*.cpp)
$(OUT)/mlk-poly: $(POLY) $(OUT)/libmlkref_patched.a
	$(CXX) $(CXXFLAGS) $(INCS) $(POLY) $(OUT)/libmlkref_patched.a -ldl -o $@

build: $(OUT)/ref_integration_check $(OUT)/mlk-poly
endif

.PHONY: all build
