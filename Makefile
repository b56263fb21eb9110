# ugdr-b200 native build: libugdr.so (client API + daemon core + sm_100a executor), the daemon,
# the smoke client, the native test and benchmark binaries.  `make -j` from the repo root;
# outputs land in ugdr_b200/_lib/ (in-tree, so they travel with the source tree).
CUDA_HOME ?= /usr/local/cuda
NVCC      := $(CUDA_HOME)/bin/nvcc
CXX       ?= g++
OUT       := ugdr_b200/_lib
OBJ       := build/obj
ARCH      := -gencode arch=compute_100a,code=sm_100a

CPPFLAGS  := -Icsrc -Iinclude -I$(CUDA_HOME)/include
CXXFLAGS  := -std=c++20 -O2 -g -fPIC -fno-semantic-interposition -Wall -Wextra -Wno-unused-parameter -pthread
NVFLAGS   := -std=c++17 $(ARCH) -O3 -lineinfo -Xcompiler -fPIC -Xptxas -v
LDLIBS    := -L$(CUDA_HOME)/lib64 -lcudart_static -ldl -lrt -lpthread

LIB_CXX := \
  csrc/common/shm.cpp csrc/queue/ring.cpp csrc/ipc/ipc.cpp \
  csrc/control/rpc.cpp csrc/control/service.cpp csrc/control/client.cpp \
  csrc/api/posting.cpp csrc/api/runtime.cpp csrc/api/memory_export.cpp \
  csrc/engine/cpu_engine.cpp csrc/gpu/cuda_memory.cpp csrc/gpu/gpu_engine.cpp csrc/gpu/diag.cpp \
  csrc/gpu/visibility.cpp csrc/gpu/trace_writer.cpp csrc/gpu/multicast.cpp \
  csrc/daemon/daemon.cpp csrc/collective/api.cpp csrc/collective/nvls.cpp \
  csrc/collective/verbs_allreduce.cpp csrc/collective/verbs_moe.cpp
LIB_CU  := csrc/gpu/executor.cu csrc/gpu/bulk_copy.cu csrc/collective/kernels.cu csrc/collective/route_noalloc.cu

LIB_OBJS := $(LIB_CXX:csrc/%.cpp=$(OBJ)/%.o) $(LIB_CU:csrc/%.cu=$(OBJ)/%.cu.o)
TEST_SRCS := $(wildcard tests/native/*.cpp)
TEST_OBJS := $(TEST_SRCS:tests/native/%.cpp=$(OBJ)/tests/%.o)

all: $(OUT)/libugdr.so $(OUT)/ugdr_daemon $(OUT)/ugdr_client $(OUT)/ugdr_native_tests $(OUT)/ugdr_perf \
     $(OUT)/ugdr_engine_bench

$(OBJ)/%.o: csrc/%.cpp
	@mkdir -p $(dir $@)
	$(CXX) $(CPPFLAGS) $(CXXFLAGS) -MMD -MP -c $< -o $@

$(OBJ)/%.cu.o: csrc/%.cu
	@mkdir -p $(dir $@)
	$(NVCC) $(CPPFLAGS) $(NVFLAGS) -MMD -MP -c $< -o $@ 2> $@.ptxas.log || (cat $@.ptxas.log; exit 1)

$(OBJ)/tests/%.o: tests/native/%.cpp
	@mkdir -p $(dir $@)
	$(CXX) $(CPPFLAGS) $(CXXFLAGS) -MMD -MP -c $< -o $@

$(OUT)/libugdr.so: $(LIB_OBJS)
	@mkdir -p $(OUT)
	$(NVCC) $(ARCH) -shared -o $@ $^ -Xlinker -soname=libugdr.so $(LDLIBS)

$(OUT)/ugdr_daemon: $(OBJ)/daemon/main.o $(OUT)/libugdr.so
	$(CXX) -o $@ $< -L$(OUT) -lugdr -Wl,-rpath,'$$ORIGIN:$$ORIGIN/../lib' -pthread

$(OUT)/ugdr_client: $(OBJ)/apps/client_main.o $(OUT)/libugdr.so
	$(CXX) -o $@ $< -L$(OUT) -lugdr -Wl,-rpath,'$$ORIGIN:$$ORIGIN/../lib' -pthread

$(OUT)/ugdr_perf: $(OBJ)/bench/ugdr_perf.o $(OUT)/libugdr.so
	$(CXX) -o $@ $< -L$(OUT) -lugdr -Wl,-rpath,'$$ORIGIN:$$ORIGIN/../lib' $(LDLIBS)

$(OUT)/ugdr_engine_bench: $(OBJ)/bench/engine_bench.o $(OUT)/libugdr.so
	$(CXX) -o $@ $< -L$(OUT) -lugdr -Wl,-rpath,'$$ORIGIN:$$ORIGIN/../lib' $(LDLIBS)

$(OUT)/ugdr_native_tests: $(TEST_OBJS) $(OUT)/libugdr.so
	$(CXX) -o $@ $(TEST_OBJS) -L$(OUT) -lugdr -Wl,-rpath,'$$ORIGIN:$$ORIGIN/../lib' $(LDLIBS)

# Sanitizer builds of the native test suite (host code instrumented; the CUDA objects are the
# regular ones): `make asan` / `make tsan`, then run build/san/<kind>/ugdr_native_tests.
SAN       := build/san
SAN_CXX   ?= /usr/bin/g++
ASAN_FLAGS := -fsanitize=address,undefined -fno-omit-frame-pointer -fno-sanitize-recover=undefined
TSAN_FLAGS := -fsanitize=thread

$(SAN)/asan/%.o: csrc/%.cpp
	@mkdir -p $(dir $@)
	$(SAN_CXX) $(CPPFLAGS) $(CXXFLAGS) $(ASAN_FLAGS) -MMD -MP -c $< -o $@
$(SAN)/asan/tests/%.o: tests/native/%.cpp
	@mkdir -p $(dir $@)
	$(SAN_CXX) $(CPPFLAGS) $(CXXFLAGS) $(ASAN_FLAGS) -MMD -MP -c $< -o $@
$(SAN)/tsan/%.o: csrc/%.cpp
	@mkdir -p $(dir $@)
	$(SAN_CXX) $(CPPFLAGS) $(CXXFLAGS) $(TSAN_FLAGS) -MMD -MP -c $< -o $@
$(SAN)/tsan/tests/%.o: tests/native/%.cpp
	@mkdir -p $(dir $@)
	$(SAN_CXX) $(CPPFLAGS) $(CXXFLAGS) $(TSAN_FLAGS) -MMD -MP -c $< -o $@

CU_OBJS := $(LIB_CU:csrc/%.cu=$(OBJ)/%.cu.o)
$(SAN)/asan/ugdr_native_tests: $(LIB_CXX:csrc/%.cpp=$(SAN)/asan/%.o) $(TEST_SRCS:tests/native/%.cpp=$(SAN)/asan/tests/%.o) $(CU_OBJS)
	$(SAN_CXX) $(ASAN_FLAGS) -o $@ $^ $(LDLIBS)
$(SAN)/tsan/ugdr_native_tests: $(LIB_CXX:csrc/%.cpp=$(SAN)/tsan/%.o) $(TEST_SRCS:tests/native/%.cpp=$(SAN)/tsan/tests/%.o) $(CU_OBJS)
	$(SAN_CXX) $(TSAN_FLAGS) -o $@ $^ $(LDLIBS)

# Whole daemons with instrumented host code (linked statically against the instrumented objects),
# for running the Python API suites against them via UGDR_DAEMON_BIN.
$(SAN)/asan/ugdr_daemon: $(LIB_CXX:csrc/%.cpp=$(SAN)/asan/%.o) $(SAN)/asan/daemon/main.o $(CU_OBJS)
	$(SAN_CXX) $(ASAN_FLAGS) -o $@ $^ $(LDLIBS)
$(SAN)/tsan/ugdr_daemon: $(LIB_CXX:csrc/%.cpp=$(SAN)/tsan/%.o) $(SAN)/tsan/daemon/main.o $(CU_OBJS)
	$(SAN_CXX) $(TSAN_FLAGS) -o $@ $^ $(LDLIBS)

asan: $(SAN)/asan/ugdr_native_tests $(SAN)/asan/ugdr_daemon
tsan: $(SAN)/tsan/ugdr_native_tests $(SAN)/tsan/ugdr_daemon

# Installed layout: $(PREFIX)/include/ugdr/*.h{,pp}, $(PREFIX)/lib/libugdr.so and ugdr.pc,
# $(PREFIX)/bin/{ugdr_daemon,ugdr_client,ugdr_perf,ugdr_engine_bench} (their rpath also looks in
# ../lib).  `make install PREFIX=/opt/ugdr`; then `pkg-config --cflags --libs ugdr`.
PREFIX ?= /usr/local
install: all
	install -d $(DESTDIR)$(PREFIX)/include/ugdr $(DESTDIR)$(PREFIX)/lib/pkgconfig $(DESTDIR)$(PREFIX)/bin
	install -m 644 include/ugdr/api.hpp include/ugdr/collective.h include/ugdr/route_noalloc.h include/ugdr/verbs_collective.h $(DESTDIR)$(PREFIX)/include/ugdr/
	install -m 755 $(OUT)/libugdr.so $(DESTDIR)$(PREFIX)/lib/
	install -m 755 $(OUT)/ugdr_daemon $(OUT)/ugdr_client $(OUT)/ugdr_perf $(OUT)/ugdr_engine_bench $(DESTDIR)$(PREFIX)/bin/
	printf 'prefix=%s\nlibdir=$${prefix}/lib\nincludedir=$${prefix}/include\n\nName: ugdr\nDescription: Userspace GPU RDMA verbs over NVLink (libibverbs-shaped C API)\nVersion: 1.0.0\nCflags: -I$${includedir}\nLibs: -L$${libdir} -Wl,-rpath,$${libdir} -lugdr\n' '$(PREFIX)' > $(DESTDIR)$(PREFIX)/lib/pkgconfig/ugdr.pc

clean:
	rm -rf build/obj build/san $(OUT)/libugdr.so $(OUT)/ugdr_daemon $(OUT)/ugdr_client $(OUT)/ugdr_native_tests $(OUT)/ugdr_perf $(OUT)/ugdr_engine_bench

-include $(shell find build/obj build/san -name '*.d' 2>/dev/null)
.PHONY: all clean asan tsan install
