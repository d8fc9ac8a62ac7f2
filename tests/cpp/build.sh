#!/bin/sh
# Builds tests/cpp/host_mirror_test against the in-tree libdeltacore.so and
# oracle/liboracle.so (both must be built first).
set -e
HERE=$(cd "$(dirname "$0")" && pwd)
ROOT=$(cd "$HERE/../.." && pwd)
CUDA=${CUDA_HOME:-/usr/local/cuda}
g++ -std=c++17 -O2 -Wall "$HERE/host_mirror_test.cpp" -o "$HERE/host_mirror_test" \
    -I"$ROOT/include" -I"$CUDA/include" \
    -L"$ROOT/burn-deltanet_b200" -ldeltacore -L"$ROOT/oracle" -loracle -L"$CUDA/lib64" -lcudart \
    -Wl,-rpath,'$ORIGIN/../../burn-deltanet_b200' -Wl,-rpath,'$ORIGIN/../../oracle' -Wl,-rpath,"$CUDA/lib64"
