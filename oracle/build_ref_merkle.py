"""Build oracle/_ref/libref_merkle.so: the reference's own Poseidon-252 Merkle layer kernel,
compiled from its source for sm_100a, with the launchers of ref_merkle_launch.inc.

It is a measuring stick, not part of the product: tests/test_ref_merkle_gpu.py checks that it
computes the same hashes as this library and bench.py times it beside this library's Merkle
kernel.  The kernel is CUDA C held in a Rust string constant (POSEIDON252_MERKLE_CUDA_KERNEL,
stwo-gpu/crates/stwo/src/prover/backend/gpu/fft.rs:2159-2946) that the reference compiles at
run time with NVRTC; this script copies that string into oracle/_ref/ (git-ignored, never
committed) and compiles it with nvcc.

Usage: python oracle/build_ref_merkle.py <reference checkout root>
"""
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: build_ref_merkle.py <reference checkout root>")
    src = Path(sys.argv[1]) / "stwo-gpu/crates/stwo/src/prover/backend/gpu/fft.rs"
    text = src.read_text()
    start = text.index('pub const POSEIDON252_MERKLE_CUDA_KERNEL: &str = r#"') 
    start = text.index('r#"', start) + 3
    end = text.index('"#;', start)
    OUT.mkdir(exist_ok=True)
    tu = OUT / "ref_merkle_tu.cu"
    tu.write_text(text[start:end] + "\n#include \"../ref_merkle_launch.inc\"\n")
    subprocess.run(["/usr/local/cuda/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo",
                    "-Xcompiler", "-fPIC", "-shared", "-o", str(OUT / "libref_merkle.so"), str(tu),
                    "-lcudart_static", "-lrt", "-lpthread", "-ldl"], check=True)
    print("built", OUT / "libref_merkle.so")


if __name__ == "__main__":
    main()
