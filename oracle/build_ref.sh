#!/usr/bin/env bash
# Builds the oracle's libraries. Test infrastructure only.
#
#   oracle/liboracle.so        the C restatement (matmulq_oracle.c), always built
#   oracle/_ref/libmtrt_ref.so the reference's own MatMulQ path, compiled from its
#                              unmodified sources where they lie, plus ref_shim.cpp
#   oracle/_ref/ref_packer_pin the reference's Golden.MatMulQ test body (its int8
#                              packer) compiled unmodified, plus ref_packer_pin.cpp
#
# The reference's CMake build needs network (FetchContent of gtest/nlohmann), so the
# few sources on the MatMulQ path are compiled directly with g++. The JSON/ONNX
# frontends, graph passes and executors are not needed by the path and are left out.
# Release flags (-DNDEBUG) as the reference's own benchmarks use; -ffp-contract=off
# keeps multiply and add separate in both libraries so they agree bit for bit.
#
# Usage: oracle/build_ref.sh [REFERENCE_ROOT]
# REFERENCE_ROOT: the argument, else $MTRTQ_REFERENCE_ROOT, else a checkout named
# "reference" beside this repository.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
REF="${1:-${MTRTQ_REFERENCE_ROOT:-${HERE}/../../reference}}"
CFLAGS="-O3 -fPIC -ffp-contract=off -fno-fast-math"

gcc ${CFLAGS} -std=c11 -shared -o "${HERE}/liboracle.so" "${HERE}/matmulq_oracle.c" -lm

if [[ ! -f "${REF}/src/ops/kernels_matmul.cpp" ]]; then
  echo "build_ref: reference sources not found under ${REF}; keeping any prebuilt _ref" >&2
  exit 0
fi

mkdir -p "${HERE}/_ref"
SRCS=(
  src/tensor/tensor.cpp
  src/ops/registry.cpp
  src/ops/kernels_matmul.cpp
  src/ops/kernels_elementwise.cpp
  src/ops/kernels_activation.cpp
  src/ops/kernels_fused.cpp
  src/ops/kernels_transformer.cpp
  src/ops/kernels_gpt.cpp
  src/graph/graph.cpp
  src/optimizer/fusion.cpp
  backends/cpu/gemm.cpp
  backends/cpu/thread_pool.cpp
)
ABS=()
for s in "${SRCS[@]}"; do ABS+=("${REF}/${s}"); done
g++ -std=c++17 ${CFLAGS} -DNDEBUG -shared -pthread \
  -I "${REF}/include" -I "${REF}" -I "${REF}/src" -I "${REF}/src/ops" \
  -o "${HERE}/_ref/libmtrt_ref.so" "${HERE}/ref_shim.cpp" "${ABS[@]}"

# The reference's own packer, run as written: its tests/golden_kernel_test.cpp,
# unmodified, against the local gtest stand-in, with the registry call and the
# goldens directory redirected (see ref_packer_pin.cpp).
g++ -std=c++17 ${CFLAGS} -DNDEBUG -pthread -c \
  -I "${HERE}/gtest_shim" -I "${REF}/include" -I "${REF}" -I "${REF}/src" -I "${REF}/src/ops" \
  -include "${HERE}/pin_prelude.h" -Dregister_builtin_kernels=pin_register_builtin_kernels \
  "-DMTRT_GOLDENS_DIR=pin_goldens_dir()" \
  -o "${HERE}/_ref/golden_kernel_test.o" "${REF}/tests/golden_kernel_test.cpp"
g++ -std=c++17 ${CFLAGS} -DNDEBUG -pthread \
  -I "${HERE}/gtest_shim" -I "${REF}/include" -I "${REF}" -I "${REF}/src" -I "${REF}/src/ops" \
  -o "${HERE}/_ref/ref_packer_pin" "${HERE}/ref_packer_pin.cpp" "${HERE}/_ref/golden_kernel_test.o" "${ABS[@]}"

# The drop-in as the reference sees it (tests/cpp/registry_drop_in.cpp): the device
# MatMulQ registered into the reference's own KernelRegistry, the reference's
# Golden.MatMulQ run through it. Needs libmtrtq.so (built first) and the CUDA runtime.
LIBDIR="${HERE}/../mini_tensorrt_b200"
CUDA_ROOT="${CUDA_HOME:-$(dirname "$(dirname "$(command -v nvcc || echo /usr/local/cuda/bin/nvcc)")")}"
if [[ -f "${LIBDIR}/libmtrtq.so" ]]; then
  g++ -std=c++17 -O2 -DNDEBUG -pthread \
    -I "${HERE}/gtest_shim" -I "${REF}/include" -I "${REF}" -I "${REF}/src" -I "${REF}/src/ops" \
    -I "${HERE}/../include" -I "${CUDA_ROOT}/include" \
    -o "${HERE}/_ref/registry_drop_in" "${HERE}/../tests/cpp/registry_drop_in.cpp" \
    "${HERE}/_ref/golden_kernel_test.o" "${ABS[@]}" \
    -L "${LIBDIR}" -lmtrtq -Wl,-rpath,'$ORIGIN/../../mini_tensorrt_b200' \
    -L "${CUDA_ROOT}/lib64" -lcudart_static -ldl -lrt
fi
echo "build_ref: built ${HERE}/liboracle.so, ${HERE}/_ref/libmtrt_ref.so, ${HERE}/_ref/ref_packer_pin and ${HERE}/_ref/registry_drop_in"
