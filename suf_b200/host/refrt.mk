# refrt.mk -- the reference's 2PC transformer-layer runtime with the B200
# engine behind proto::make_real_gpu_backend(), wired as a maintainer would
# wire the drop-in: the reference's nn/ runtime/ compiler/ sources (compiled
# where they lie in the reference checkout; nothing is copied), this
# package's adapter (make_backend.cpp), its launch_* shim of the reference's
# cuda_primitives ABI and libsufb200.so.  Output: suf_b200/_refrt/.
#   make -f suf_b200/host/refrt.mk REF=<reference checkout> [-j8]
#   _refrt/layer_harness_b200  layer_harness.cpp on the B200 engine
#   _refrt/ops_harness_b200    ops_harness.cpp (the hot-path operations through
#                              the reference's backend interfaces) on it
# suf_b200.build runs it when a reference checkout is present.
REF ?=
HOSTDIR := $(dir $(abspath $(lastword $(MAKEFILE_LIST))))
PKG := $(abspath $(HOSTDIR)..)
REPO := $(abspath $(PKG)/..)
OUT := $(PKG)/_refrt
CUDA ?= /usr/local/cuda

CXXFLAGS := -std=gnu++20 -O2 -fopenmp -fPIC -DSUF_HAVE_CUDA=1 -DSUFB200_WITH_REFERENCE_PROTO \
            -I$(REF)/include -I$(REF)/cuda -I$(REPO)/include -I$(HOSTDIR) -I$(CUDA)/include -w
NVFLAGS := -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -DSUF_HAVE_CUDA=1 \
           -Xcompiler -fPIC,-fopenmp -I$(REF)/include -I$(REF)/cuda -w

# The reference runtime of the layer (the sources of its nn_ops and
# compiler_passes libraries, CMakeLists.txt:277-343, without matmul_gpu.cu).
RT := nn/linops nn/matmul_publicW nn/matmul_beaver nn/attention_block nn/mlp_block nn/transformer_layer \
      nn/model_specs gates/postproc_hooks runtime/bench_accounting runtime/pfss_superbatch \
      runtime/open_collector runtime/phase_executor runtime/pfss_gpu_stager_cuda \
      compiler/truncation_pass compiler/rescale_pass compiler/layer_graph compiler/suf_to_pfss
RT_OBJ := $(patsubst %,$(OUT)/rt/%.o,$(RT))
OURS := $(OUT)/ours/make_backend.o $(OUT)/ours/cuda_primitives_shim.o $(OUT)/ours/matmul_gpu.o

.PHONY: all need-ref
all: need-ref $(OUT)/layer_harness_b200 $(OUT)/ops_harness_b200

need-ref:
	@test -n "$(REF)" -a -d "$(REF)/src/nn" || { echo "set REF=<reference checkout>" >&2; exit 2; }

$(OUT)/rt/%.o: $(REF)/src/%.cpp
	@mkdir -p $(dir $@)
	g++ $(CXXFLAGS) -c $< -o $@

$(OUT)/ours/%.o: $(HOSTDIR)%.cpp $(HOSTDIR)sufb200_backend.hpp
	@mkdir -p $(dir $@)
	g++ $(CXXFLAGS) -c $< -o $@

# the reference's public-weight matmul (src/nn/matmul_gpu.cu): part of its nn
# layer, not of the PFSS backend
$(OUT)/ours/matmul_gpu.o: $(REF)/src/nn/matmul_gpu.cu
	@mkdir -p $(dir $@)
	$(CUDA)/bin/nvcc $(NVFLAGS) -c $< -o $@

$(OUT)/layer_harness_b200: $(OUT)/ours/layer_harness.o $(RT_OBJ) $(OURS) $(PKG)/libsufb200.so
	g++ -fopenmp -o $@ $(OUT)/ours/layer_harness.o $(RT_OBJ) $(OURS) -L$(PKG) -lsufb200 \
	    -L$(CUDA)/lib64 -lcudart -lcrypto -Wl,-rpath,'$$ORIGIN/..'

$(OUT)/ops_harness_b200: $(OUT)/ours/ops_harness.o $(RT_OBJ) $(OURS) $(PKG)/libsufb200.so
	g++ -fopenmp -o $@ $(OUT)/ours/ops_harness.o $(RT_OBJ) $(OURS) -L$(PKG) -lsufb200 \
	    -L$(CUDA)/lib64 -lcudart -lcrypto -Wl,-rpath,'$$ORIGIN/..'
