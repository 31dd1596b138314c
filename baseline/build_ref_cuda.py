"""Build the reference's own CUDA extension for sm_100a into baseline/_ref/.

The reference (flurinh/RapidAlign) ships its GPU path as a PyTorch extension
of two source files, csrc/bindings.cpp and csrc/kde_similarity.cu.  This
recipe compiles those files, unmodified and where they lie in a checkout of
the reference, with torch.utils.cpp_extension and flags of its own (not the
reference's setup.py): -O3 and -gencode arch=compute_100a,code=sm_100a.  The
module it leaves in baseline/_ref/ (git-ignored; built files travel with the
repository to the machine that runs the bench) is what
`bench.py --impl reference-gpu` times: the reference's segmented forward and
backward kernels on the benchmark's batch.

    python baseline/build_ref_cuda.py [--ref PATH_TO_REFERENCE_CHECKOUT]
"""
import argparse
import glob
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NAME = "rapidalign_ref_cuda"


def built_module() -> str:
    """Path of the built module, or '' when it is not there."""
    hits = sorted(glob.glob(os.path.join(OUT, NAME + "*.so")))
    return hits[0] if hits else ""


def build(ref: str = "/root/reference", force: bool = False) -> str:
    if built_module() and not force:
        return built_module()
    src = [os.path.join(ref, "csrc", "bindings.cpp"), os.path.join(ref, "csrc", "kde_similarity.cu")]
    for s in src:
        if not os.path.exists(s):
            raise FileNotFoundError(s)
    from torch.utils import cpp_extension
    os.makedirs(OUT, exist_ok=True)
    cpp_extension.load(
        name=NAME, sources=src, build_directory=OUT, verbose=False,
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        extra_include_paths=[os.path.join(ref, "csrc")])
    return built_module()


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    path = build(a.ref, a.force)
    print(path)
    sys.exit(0 if path else 1)
