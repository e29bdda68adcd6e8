"""Makes the reference's own harness (src/main.cu) run on this library.

Built against include/reference_compat/ (kernels.cuh, quant.cuh over
int4gemm.hpp and libi4g.so), the harness compiles unmodified. One contract
differs: launch_final reads this library's sm_100a tile layout
(launch_repack_umma) where the reference's final kernel read the mma.sync
lane-native layouts (src/main.cu:216-220, 322-329). This script writes a copy
of main.cu with the one change a maintainer makes for that: after the harness
has checked its reference layouts byte for byte (validate_repack), the
buffers it hands to "final" (and to launch_final_fp32) are refilled with the
tile layout, and the one-shot row repacks into the tile layout. Every edit is
an exact match that must occur once; the script fails loudly otherwise.

    python3 harness_patch.py <reference>/src/main.cu <out.cu>
"""
import sys

HELPER = """// [i4g] launch_final here reads the sm_100a tile layout (launch_repack_umma):
// refill the buffers the harness passes to "final" and launch_final_fp32.
void use_tile_layout(CaseBuffers& x) {
  launch_repack_umma(x.packed.get(), x.mma_repacked.get(), x.K, x.N);
  launch_repack_umma(x.packed.get(), x.mma_pair_repacked.get(), x.K, x.N);
  launch_repack_umma(x.packed.get(), x.repacked.get(), x.K, x.N);
  CUDA_CHECK(cudaDeviceSynchronize());
}

"""

# (anchor, replacement): the anchor text must occur exactly once
EDITS = [
    # the helper, ahead of the layout-choosing predicates
    ("bool uses_mma_repack(", HELPER + "bool uses_mma_repack("),
    # correctness(): after the reference layouts are validated
    ("  CaseBuffers x(size, size, size, group);\n  validate_repack(x);\n",
     "  CaseBuffers x(size, size, size, group);\n  validate_repack(x);\n  use_tile_layout(x);\n"),
    # fp32_output_check()
    ("validate_repack(x); CublasHandle blas;",
     "validate_repack(x); use_tile_layout(x); CublasHandle blas;"),
    # benchmark_all(): the one-shot row repacks into the tile layout
    ("        launch_repack_mma_pair_128x32(x.packed.get(),x.mma_pair_repacked.get(),K,N);",
     "        launch_repack_umma(x.packed.get(),x.mma_pair_repacked.get(),K,N);"),
    ("        launch_repack_mma_128x32(x.packed.get(),x.mma_repacked.get(),K,N);",
     "        launch_repack_umma(x.packed.get(),x.mma_repacked.get(),K,N);"),
    # benchmark_all(): after the preprocessing rows, before the registry loop
    ("    cublas_row_gemm(blas.h,x.a.get(),x.dequant.get(),x.reference.get(),M,N,K);",
     "    use_tile_layout(x);\n"
     "    cublas_row_gemm(blas.h,x.a.get(),x.dequant.get(),x.reference.get(),M,N,K);"),
    # profile_one()
    ("  CaseBuffers x(size,size,size,group);\n  for (auto& entry:kernel_registry())",
     "  CaseBuffers x(size,size,size,group);\n  use_tile_layout(x);\n"
     "  for (auto& entry:kernel_registry())"),
]


def patch(text: str) -> str:
    for anchor, new in EDITS:
        n = text.count(anchor)
        if n != 1:
            raise SystemExit(f"harness_patch: expected one match of {anchor[:60]!r}, found {n}")
        text = text.replace(anchor, new)
    return text


def main(argv):
    if len(argv) != 3:
        raise SystemExit(__doc__)
    with open(argv[1]) as f:
        src = f.read()
    with open(argv[2], "w") as f:
        f.write(patch(src))


if __name__ == "__main__":
    main(sys.argv)
