# voltattn_b200 build: the C-ABI library (sm_100a), the CLI, and the test-only
# oracle (oracle/Makefile). `python -c "import __graft_entry__ as g; g.build()"`
# runs the same steps.
NVCC      ?= nvcc
ARCH      := -gencode arch=compute_100a,code=sm_100a
NVFLAGS   := -O3 -std=c++17 -lineinfo $(ARCH) -Xcompiler -fPIC,-Wall,-Wextra -Xptxas -v --expt-relaxed-constexpr
CSRC      := voltattn_b200/csrc
HDRS      := $(wildcard $(CSRC)/*.cuh) include/voltattn.h include/voltattn.hpp
LIB       := voltattn_b200/libvoltattn_b200.so
CLI       := voltattn_b200/bin/voltattn

all: $(LIB) $(CLI) oracle

$(LIB): $(CSRC)/voltattn_api.cu $(HDRS)
	$(NVCC) $(NVFLAGS) -shared -o $@ $(CSRC)/voltattn_api.cu 2> voltattn_b200/ptxas.log || (cat voltattn_b200/ptxas.log; false)

$(CLI): $(CSRC)/cli/voltattn_main.cu $(LIB) $(HDRS)
	@mkdir -p voltattn_b200/bin
	$(NVCC) -O3 -std=c++17 $(ARCH) -o $@ $(CSRC)/cli/voltattn_main.cu -Lvoltattn_b200 -lvoltattn_b200 \
	  -Xlinker -rpath,'$$ORIGIN/..'

oracle:
	$(MAKE) -C oracle

clean:
	rm -f $(LIB) $(CLI) voltattn_b200/ptxas.log

.PHONY: all oracle clean
