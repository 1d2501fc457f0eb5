# `make lib`: the shared library a reference caller builds and loads through
# ctypes (the reference's Makefile:29-33 `lib` target and
# host/launcher.py:103-132 compile_shared_library produce megakernel.so).
# Here it is built for sm_100a only (B200), from this repository's sources;
# it exports the same six reference symbols plus the extensions declared in
# include/megakernel.h.  `make package-lib` builds the copy the Python
# package loads (megakernel_b200/libmegakernel.so); both are the same code.

NVCC ?= nvcc
ARCH_FLAGS = -gencode arch=compute_100a,code=sm_100a
NVCC_FLAGS = -O3 -std=c++17 -lineinfo -Xcompiler -fPIC
CSRC = megakernel_b200/csrc
UNITS = $(CSRC)/megakernel.cu $(CSRC)/tp.cu
DEPS = $(wildcard $(CSRC)/*.cu $(CSRC)/*.cuh) include/megakernel.h
BUILD ?= _build
LIB_OUT ?= megakernel.so

.PHONY: lib package-lib clean

lib: $(LIB_OUT)

package-lib: megakernel_b200/libmegakernel.so

$(BUILD)/%.o: $(CSRC)/%.cu $(DEPS)
	@mkdir -p $(BUILD)
	$(NVCC) $(ARCH_FLAGS) $(NVCC_FLAGS) -c $< -o $@

$(LIB_OUT) megakernel_b200/libmegakernel.so: $(BUILD)/megakernel.o $(BUILD)/tp.o
	$(NVCC) $(ARCH_FLAGS) -shared $^ -o $@

clean:
	rm -rf $(BUILD) $(LIB_OUT)
