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

# One translation unit per kernel family, compiled in parallel as
# relocatable device code (one device error word shared by all of them) and
# device-linked into the shared library.
SRCS      := $(CSRC)/voltattn_api.cu $(CSRC)/host_util.cu $(CSRC)/launch_tc.cu $(CSRC)/launch_tcg.cu \
             $(CSRC)/launch_mma.cu $(CSRC)/launch_prefill.cu $(CSRC)/launch_stream_g1.cu \
             $(CSRC)/launch_stream_g2.cu $(CSRC)/launch_stream_g4.cu $(CSRC)/launch_stream_g8.cu
OBJDIR    := voltattn_b200/_build
OBJS      := $(patsubst $(CSRC)/%.cu,$(OBJDIR)/%.o,$(SRCS))

$(OBJDIR)/%.o: $(CSRC)/%.cu $(HDRS) $(wildcard $(CSRC)/*.cuh)
	@mkdir -p $(OBJDIR)
	$(NVCC) $(NVFLAGS) -rdc=true -c -o $@ $< 2> $@.log || (cat $@.log; false)

$(LIB): $(OBJS)
	$(NVCC) $(ARCH) -shared -rdc=true -o $@ $(OBJS) -lcuda 2> voltattn_b200/link.log || (cat voltattn_b200/link.log; false)
	cat $(OBJDIR)/*.o.log > voltattn_b200/ptxas.log

$(CLI): $(CSRC)/cli/voltattn_main.cu $(LIB) $(HDRS)
	@mkdir -p voltattn_b200/bin
	$(NVCC) -O3 -std=c++17 $(ARCH) -o $@ $(CSRC)/cli/voltattn_main.cu -Lvoltattn_b200 -lvoltattn_b200 \
	  -Xlinker -rpath,'$$ORIGIN/..'

# Development build with the tile kernel's per-CTA %globaltimer timeline
# (-DVA_TC_TIMELINE), used by `python bench.py --timeline`; not the product.
TLDIR     := voltattn_b200/_build/timeline
timeline: $(OBJS)
	@mkdir -p $(TLDIR)/voltattn_b200
	$(NVCC) $(NVFLAGS) -rdc=true -DVA_TC_TIMELINE -c -o $(TLDIR)/launch_tc.o $(CSRC)/launch_tc.cu 2> $(TLDIR)/ptxas.log
	$(NVCC) $(ARCH) -shared -rdc=true -o $(TLDIR)/voltattn_b200/libvoltattn_b200.so \
	  $(filter-out $(OBJDIR)/launch_tc.o,$(OBJS)) $(TLDIR)/launch_tc.o -lcuda
	cp voltattn_b200/__init__.py voltattn_b200/launcher.py $(TLDIR)/voltattn_b200/

oracle:
	$(MAKE) -C oracle REF_SRC="$(REF_SRC)"

clean:
	rm -rf $(LIB) $(CLI) voltattn_b200/ptxas.log voltattn_b200/link.log $(OBJDIR)

.PHONY: all oracle clean timeline
