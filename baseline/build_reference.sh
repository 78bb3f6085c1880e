#!/bin/bash
# Builds the unmodified tiny-nccl reference with its own CMake project and
# installs the artefacts under baseline/_ref (git-ignored):
#   lib/libtiny_nccl.a        the reference's static library, as CMake built it
#   lib/libtiny_nccl_ref.so   the same archive linked whole into a shared object
#                             (static cudart) so Python can load it with ctypes
#   bin/tnccl_allreduce       the reference's example launcher
#   bin/tnccl_ring_model_test the reference's CPU model test
# `pip install --target baseline/_ref <reference>` cannot work: the reference
# has neither setup.py nor pyproject.toml. Its CMakeLists.txt accepts only
# numeric CMAKE_CUDA_ARCHITECTURES, so "100a" is refused and "100" (sm_100,
# which runs on B200) is used.
#
#   baseline/build_reference.sh <reference source directory>
set -euo pipefail
if [ $# -ne 1 ]; then
  echo "usage: $0 <reference source directory>" >&2
  exit 2
fi
SRC=$1
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="$HERE/_ref"
WORK=$(mktemp -d /tmp/tnccl_ref.XXXXXX)
cp -r "$SRC" "$WORK/src"
cmake -S "$WORK/src" -B "$WORK/build" -DCMAKE_BUILD_TYPE=Release -DTNCCL_BUILD_CUDA=ON \
  -DTNCCL_BUILD_EXAMPLES=ON -DTNCCL_BUILD_TESTS=ON -DCMAKE_CUDA_ARCHITECTURES=100
cmake --build "$WORK/build" -j8
mkdir -p "$OUT/lib" "$OUT/bin" "$OUT/include"
cp "$WORK/build/libtiny_nccl.a" "$OUT/lib/"
cp "$WORK/build/tnccl_allreduce" "$WORK/build/tnccl_ring_model_test" "$OUT/bin/"
cp "$WORK/src/include/tnccl.h" "$OUT/include/"
g++ -shared -o "$OUT/lib/libtiny_nccl_ref.so" -Wl,--whole-archive "$OUT/lib/libtiny_nccl.a" \
  -Wl,--no-whole-archive -L/usr/local/cuda/lib64 -lcudart_static -ldl -lrt -lpthread
"$OUT/bin/tnccl_ring_model_test"
rm -rf "$WORK"
echo "reference installed in $OUT"
