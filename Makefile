# FlashGANN-B200 build.
#
#   make gpu_flashgann [EXTRA_NVFLAGS="-DINTERNAL_TOPK=1024"]   -> bin/gpu_flashgann (+ the library)
#   make lib                                                  -> flashgann_b200/libflashgann.so
#   make oracle                                               -> oracle/liboracle.so (test infrastructure)
#
# Same knobs as the reference Makefile (ARCH, EXTRA_NVFLAGS); this build
# targets sm_100a only.
NVCC    ?= nvcc
ARCH    ?= sm_100a
GENCODE := -gencode arch=compute_100a,code=$(ARCH)
NVFLAGS := -std=c++17 -O3 $(GENCODE) -lineinfo -Xptxas -v $(EXTRA_NVFLAGS)
CSRC    := flashgann_b200/csrc
LIB     := flashgann_b200/libflashgann.so
BIN_DIR := bin

KERNEL_SRC := $(CSRC)/fg_search.cu $(CSRC)/fg_search_warp.cu $(CSRC)/fg_shard_merge.cu $(CSRC)/fg_api.cu
HEADERS    := $(CSRC)/fg_config.h $(CSRC)/fg_internal.h $(CSRC)/fg_device.cuh include/flashgann.h
OBJ_DIR    := flashgann_b200/_build
OBJS       := $(patsubst $(CSRC)/%.cu,$(OBJ_DIR)/%.o,$(KERNEL_SRC))

.PHONY: all lib gpu_flashgann oracle clean

all: lib gpu_flashgann

lib: $(LIB)

$(OBJ_DIR)/%.o: $(CSRC)/%.cu $(HEADERS) | $(OBJ_DIR)
	$(NVCC) $(NVFLAGS) -Xcompiler -fPIC -c -o $@ $< 2> $(OBJ_DIR)/$*.ptxas.log || (cat $(OBJ_DIR)/$*.ptxas.log; exit 1)

$(OBJ_DIR):
	mkdir -p $(OBJ_DIR)

$(LIB): $(OBJS)
	$(NVCC) $(GENCODE) -shared -o $@ $(OBJS)
	cat $(OBJ_DIR)/*.ptxas.log > $(CSRC)/ptxas.log

$(BIN_DIR):
	mkdir -p $(BIN_DIR)

gpu_flashgann: $(BIN_DIR)/gpu_flashgann

# nvcc drives the host compiler for the CLI too, as the reference's Makefile
# does for main.cu, so every EXTRA_NVFLAGS a reference build accepts
# (-DINTERNAL_TOPK=..., -Xptxas ..., -Xcompiler ...) is valid here as well
$(BIN_DIR)/gpu_flashgann: $(CSRC)/fg_cli.cpp $(LIB) | $(BIN_DIR)
	$(NVCC) $(NVFLAGS) -o $@ $(CSRC)/fg_cli.cpp -L$(dir $(LIB)) -lflashgann -Xlinker -rpath,'$$ORIGIN/../flashgann_b200'

oracle:
	$(MAKE) -C oracle

clean:
	rm -f $(LIB) $(BIN_DIR)/gpu_flashgann $(CSRC)/ptxas.log $(OBJS) $(OBJ_DIR)/*.ptxas.log
