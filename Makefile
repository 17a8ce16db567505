# Builds the B200 attention library and its checkers.
#   make            -> tinyllama-engine_b200/libtle_attn.so (nvcc, sm_100a) + oracle
#   make oracle     -> oracle/liboracle.so and, when the reference tree is
#                      present, oracle/_ref/libref_attn.so
#   make cpptest    -> tests/cpp/test_ops_gpu (reference-style tests via the C++ shim)
CUDA_HOME ?= /usr/local/cuda
NVCC ?= $(CUDA_HOME)/bin/nvcc
CXX := g++
PKG := tinyllama-engine_b200
CSRC := $(PKG)/csrc
HOST := $(PKG)/host
LIB := $(PKG)/libtle_attn.so
# Reference checkout for oracle/_ref: by default the one beside this repository.
REF ?= $(abspath $(CURDIR)/../reference)

ARCH := -gencode arch=compute_100a,code=sm_100a
NVFLAGS := -std=c++20 -O3 $(ARCH) -lineinfo -Xcompiler -fPIC -Xcompiler -Wall \
           --expt-relaxed-constexpr -Iinclude -I$(CSRC)
CU_SRCS := $(CSRC)/decode.cu $(CSRC)/decode_bf16.cu $(CSRC)/prefill.cu $(CSRC)/forward.cu $(CSRC)/gemm.cu \
           $(CSRC)/abi.cu
HOST_SRCS := $(HOST)/ops_gpu.cpp
CU_OBJS := $(patsubst $(CSRC)/%.cu,_build/%.o,$(CU_SRCS))
HOST_OBJS := $(patsubst $(HOST)/%.cpp,_build/host_%.o,$(HOST_SRCS))

all: $(LIB) oracle cpptest

_build:
	mkdir -p _build

_build/%.o: $(CSRC)/%.cu $(CSRC)/common.cuh $(CSRC)/tcgen05.cuh $(CSRC)/kernels.h include/tle_attn.h include/tle_forward.h | _build
	$(NVCC) $(NVFLAGS) -c $< -o $@

_build/host_%.o: $(HOST)/%.cpp $(HOST)/ops_gpu.h include/tle_attn.h include/tle_forward.h | _build
	$(CXX) -std=c++20 -O2 -g -Wall -Wextra -fPIC -Iinclude -I$(CUDA_HOME)/include -c $< -o $@

$(LIB): $(CU_OBJS) $(HOST_OBJS)
	$(NVCC) $(ARCH) -shared $^ -o $@

oracle:
	$(MAKE) -C oracle REF=$(REF)

cpptest: tests/cpp/test_ops_gpu

tests/cpp/test_ops_gpu: $(LIB) tests/cpp/test_ops_gpu.cpp $(HOST)/ops_gpu.h include/tle_forward.h
	g++ -std=c++20 -O2 -Wall -Iinclude -I$(HOST) tests/cpp/test_ops_gpu.cpp \
	    -L$(PKG) -ltle_attn -Wl,-rpath,'$$ORIGIN/../../$(PKG)' -o tests/cpp/test_ops_gpu

ptxas-info:
	$(NVCC) $(NVFLAGS) -Xptxas -v -c $(CSRC)/decode.cu -o /dev/null
	$(NVCC) $(NVFLAGS) -Xptxas -v -c $(CSRC)/prefill.cu -o /dev/null
	$(NVCC) $(NVFLAGS) -Xptxas -v -c $(CSRC)/forward.cu -o /dev/null

clean:
	rm -rf _build $(LIB) tests/cpp/test_ops_gpu
	$(MAKE) -C oracle clean

.PHONY: all oracle cpptest ptxas-info clean
