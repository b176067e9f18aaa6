#!/usr/bin/env bash
# Test infrastructure only: compiles the UNMODIFIED reference Jasper FFI
# library (ffi/*.cu + include/jasper/**) from the read-only reference tree,
# for sm_100a, into oracle/_ref/lib/libjasper_ffi.so.  It is the GPU-side
# oracle for search/build parity and the `bench.py --impl reference` arm.
# The reference's CMake build cannot run offline (CPM fetches from GitHub,
# CMakeLists.txt:27-55), so the same flags are passed to nvcc directly:
#   -rdc=true -lineinfo (CMakeLists.txt:19), JASPER_STABLE_IDS=0 and
#   JASPER_ENABLE_COMPACT=0 (the shipped defaults, graph.cuh:29-34), no NDEBUG
#   (device asserts stay on, as in the reference's default build type).
# Usage: oracle/build_ref.sh REFERENCE_ROOT
set -euo pipefail
REF=${1:?usage: oracle/build_ref.sh REFERENCE_ROOT}
HERE=$(cd "$(dirname "$0")" && pwd)
OUT=$HERE/_ref
TVM=$(python -c "import tvm_ffi,os;print(os.path.dirname(tvm_ffi.__file__))")
mkdir -p "$OUT/obj" "$OUT/lib"
FLAGS="-std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -rdc=true -lineinfo \
  --extended-lambda --expt-relaxed-constexpr -Xcompiler -fPIC \
  -DJASPER_STABLE_IDS=0 -DJASPER_ENABLE_COMPACT=0 \
  -I$REF/include -I$TVM/include"
TUS=${JASPER_REF_TUS:-"plain directional_l2_k4 directional_l2_k16 directional_ip_k4 directional_ip_k16"}
pids=()
for tu in $TUS; do
  src=$REF/ffi/jasper_ffi_$tu.cu
  obj=$OUT/obj/$tu.o
  if [ ! -f "$obj" ] || [ "$src" -nt "$obj" ]; then
    nvcc $FLAGS -c "$src" -o "$obj" > "$OUT/obj/$tu.log" 2>&1 &
    pids+=($!)
  fi
done
for p in "${pids[@]:-}"; do [ -n "$p" ] && wait "$p"; done
objs=""
for tu in $TUS; do objs="$objs $OUT/obj/$tu.o"; done
nvcc -gencode arch=compute_100a,code=sm_100a -dlink -Xcompiler -fPIC $objs -o "$OUT/obj/dlink.o"
g++ -shared -o "$OUT/lib/libjasper_ffi.so" $objs "$OUT/obj/dlink.o" \
  -L/usr/local/cuda/lib64 -lcudart -lcublas -lcurand \
  -L$TVM/lib -ltvm_ffi -Wl,-rpath,$TVM/lib -Wl,-rpath,/usr/local/cuda/lib64
echo "built $OUT/lib/libjasper_ffi.so"
# The same plain-graph ops built with -DNDEBUG (device asserts compiled out):
# a second, stricter reference bar for the benchmark (bench.py --ref-ndebug).
NDOBJ=$OUT/obj/plain_ndebug.o
if [ ! -f "$NDOBJ" ] || [ "$REF/ffi/jasper_ffi_plain.cu" -nt "$NDOBJ" ]; then
  nvcc $FLAGS -DNDEBUG -c "$REF/ffi/jasper_ffi_plain.cu" -o "$NDOBJ" > "$OUT/obj/plain_ndebug.log" 2>&1
fi
nvcc -gencode arch=compute_100a,code=sm_100a -dlink -Xcompiler -fPIC "$NDOBJ" -o "$OUT/obj/dlink_ndebug.o"
g++ -shared -o "$OUT/lib/libjasper_ffi_ndebug.so" "$NDOBJ" "$OUT/obj/dlink_ndebug.o" \
  -L/usr/local/cuda/lib64 -lcudart -lcublas -lcurand \
  -L$TVM/lib -ltvm_ffi -Wl,-rpath,$TVM/lib -Wl,-rpath,/usr/local/cuda/lib64
echo "built $OUT/lib/libjasper_ffi_ndebug.so"
# RaBitQ quantizer driver (header-only reference code; our main() in
# oracle/ref_rabitq_driver.cu)
mkdir -p "$OUT/bin"
if [ ! -f "$OUT/bin/ref_rabitq" ] || [ "$HERE/ref_rabitq_driver.cu" -nt "$OUT/bin/ref_rabitq" ]; then
  nvcc -std=c++17 -O3 -gencode arch=compute_100a,code=sm_100a -lineinfo --expt-relaxed-constexpr \
    -I$REF/include "$HERE/ref_rabitq_driver.cu" -o "$OUT/bin/ref_rabitq" -lcublas -lcurand
fi
echo "built $OUT/bin/ref_rabitq"
