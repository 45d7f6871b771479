# Build recipe for the UNMODIFIED reference FlashTrie (Dakshitha-BA/flash-trie)
# from its own sources, without running the reference's CMake build.
#
# Test infrastructure only: the result is the reference's pybind11 module,
# renamed to `flashtrie_ref` at compile time so it can sit beside this
# project's own `flashtrie` module.  It is used to generate golden vectors
# (tests/golden/make_golden.py) and as the timed CPU baseline
# (`bench.py --impl reference`).  Nothing in the product links or imports it.
#
#   make -f oracle/ref.mk REF=/path/to/reference        (from the repo root)
#
# REF defaults to $(FT_REFERENCE), the environment variable __graft_entry__
# and tests/golden/make_golden.py also read.
#
# Output (git-ignored, travels to the GPU box):
#   oracle/_ref/flashtrie_ref$(EXT)  the reference's pybind11 module
#   oracle/_ref/marisa-lookup        the reference's key-id lookup tool
#   oracle/_ref/ref_build            oracle/ref_build.cc over the reference's
#                                    builder (Keyset + Trie::build + save)
#
# Flags follow the reference's CMakeLists.txt:21-27 (MARISA_USE_POPCNT,
# MARISA_USE_BMI2, -mpopcnt -mbmi2) except -march=native, since the module is
# built here and run on another x86-64 host.  MARISA_USE_BMI2 is required for
# the GPU path: without it the device-side select0 would call the host-only
# table version of select_bit (bit-vector.cc:18-31 vs :33-392).

REF      ?= $(FT_REFERENCE)
OUT      := oracle/_ref
OBJ      := $(OUT)/obj
PYINC    := $(shell python3 -c "import sysconfig;print(sysconfig.get_paths()['include'])")
PYBIND   := $(shell python3 -c "import pybind11;print(pybind11.get_include())")
EXT      := $(shell python3 -c "import sysconfig;print(sysconfig.get_config_var('EXT_SUFFIX'))")
NVCC     ?= nvcc
CXX      := /usr/bin/g++
ARCH     := -gencode arch=compute_100a,code=sm_100a
INCS     := -I$(REF)/include -I$(REF)/lib -I/usr/local/cuda/include
DEFS     := -DMARISA_USE_POPCNT -DMARISA_USE_BMI2 -DNDEBUG
HOSTFL   := -O3 -std=c++17 -fPIC -fopenmp -mpopcnt -mbmi2 -w
CUFLAGS  := -O3 -std=c++17 -rdc=true --expt-relaxed-constexpr -lineinfo $(ARCH) \
            -ccbin $(CXX) -Xcompiler -fPIC,-fopenmp,-mpopcnt,-mbmi2,-O3,-w $(INCS) $(DEFS)
CXXFLAGS := $(HOSTFL) $(INCS) $(DEFS)

CU_SRCS  := lib/marisa/grimoire/trie/louds-trie.cc lib/marisa/grimoire/trie/tail.cc \
            lib/marisa/grimoire/vector/bit-vector.cc
CXX_SRCS := lib/marisa/keyset.cc lib/marisa/agent.cc lib/marisa/trie.cc \
            lib/marisa/grimoire/io/mapper.cc lib/marisa/grimoire/io/reader.cc \
            lib/marisa/grimoire/io/writer.cc
CU_OBJS  := $(patsubst %.cc,$(OBJ)/%.o,$(CU_SRCS))
CXX_OBJS := $(patsubst %.cc,$(OBJ)/%.o,$(CXX_SRCS))
BIND_OBJ := $(OBJ)/tools/bindings.o
DLINK    := $(OBJ)/dlink.o
MODULE   := $(OUT)/flashtrie_ref$(EXT)
# The reference's own key-id lookup tool (tools/marisa-lookup.cc): pins the
# key ids the engine reports against the reference's LoudsTrie::lookup.
LOOKUP   := $(OUT)/marisa-lookup
TOOL_OBJS := $(OBJ)/tools/marisa-lookup.o $(OBJ)/tools/cmdopt.o

# The reference's own builder driven from flat key files (oracle/ref_build.cc):
# the reference arm of bench.py builds its trie with it.
REFBUILD := $(OUT)/ref_build
REFBUILD_OBJ := $(OBJ)/ref_build.o

all: $(MODULE) $(LOOKUP) $(REFBUILD)

ifeq ($(strip $(REF)),)
$(error REF is empty: pass REF=/path/to/reference or set FT_REFERENCE)
endif

$(CU_OBJS): $(OBJ)/%.o: $(REF)/%.cc
	@mkdir -p $(dir $@)
	$(NVCC) $(CUFLAGS) -x cu -c $< -o $@

$(CXX_OBJS): $(OBJ)/%.o: $(REF)/%.cc
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -c $< -o $@

# The module name is a token in bindings.cpp (PYBIND11_MODULE(flashtrie, m));
# -Dflashtrie=flashtrie_ref renames it without touching the source.
$(BIND_OBJ): $(REF)/tools/bindings.cpp
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -Dflashtrie=flashtrie_ref -I$(REF)/tools -I$(PYINC) -I$(PYBIND) -c $< -o $@

$(DLINK): $(CU_OBJS)
	$(NVCC) $(ARCH) -Xcompiler -fPIC -dlink $^ -o $@

$(MODULE): $(CU_OBJS) $(CXX_OBJS) $(BIND_OBJ) $(DLINK)
	$(CXX) -shared -fopenmp -o $@ $^ -L/usr/local/cuda/lib64 -lcudart -Wl,-rpath,/usr/local/cuda/lib64

$(TOOL_OBJS): $(OBJ)/tools/%.o: $(REF)/tools/%.cc
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -I$(REF)/tools -c $< -o $@

$(LOOKUP): $(CU_OBJS) $(CXX_OBJS) $(TOOL_OBJS) $(DLINK)
	$(CXX) -fopenmp -o $@ $^ -L/usr/local/cuda/lib64 -lcudart -Wl,-rpath,/usr/local/cuda/lib64

$(REFBUILD_OBJ): oracle/ref_build.cc
	@mkdir -p $(dir $@)
	$(CXX) $(CXXFLAGS) -c $< -o $@

$(REFBUILD): $(CU_OBJS) $(CXX_OBJS) $(REFBUILD_OBJ) $(DLINK)
	$(CXX) -fopenmp -o $@ $^ -L/usr/local/cuda/lib64 -lcudart -Wl,-rpath,/usr/local/cuda/lib64

clean:
	rm -rf $(OUT)

.PHONY: all clean
