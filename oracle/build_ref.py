"""Build recipe for oracle/_ref/ -- the reference's OWN fp32 scalar GDN kernel, compiled from its
source where it lies (kernels/qwen35moe_gdn_prefill.cu of the reference checkout) for sm_100a.

TEST INFRASTRUCTURE ONLY.  The resulting torch extension is run on a B200 to produce the golden
GDN outputs under tests/golden/ that pin the C restatement in oracle/gdn_recurrent.c.  It uses
the reference's own compile flags (kernels/qwen35moe_gdn_prefill.py:49-61) with the target
architecture changed from sm_89 to sm_100a.  Nothing is copied out of the reference tree.

    python oracle/build_ref.py [--reference /path/to/reference]
"""

from __future__ import annotations

import argparse
import importlib.util
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref" / "gdn_scalar"
NAME = "ref_gdn_scalar"
DEFAULT_REFERENCE = pathlib.Path("/root/reference")


def build(reference: pathlib.Path = DEFAULT_REFERENCE) -> pathlib.Path:
    from torch.utils.cpp_extension import load

    src = reference / "kernels" / "qwen35moe_gdn_prefill.cu"
    if not src.exists():
        raise FileNotFoundError(src)
    OUT.mkdir(parents=True, exist_ok=True)
    load(name=NAME, sources=[str(src)], build_directory=str(OUT), verbose=False,
         extra_cflags=["-O3", "-std=c++17", "-w"],
         extra_cuda_cflags=["-O3", "-lineinfo", "-w", "--use_fast_math", "-std=c++17", "--expt-relaxed-constexpr",
                            "--expt-extended-lambda", "-gencode=arch=compute_100a,code=sm_100a"])
    return OUT / f"{NAME}.so"


def load_built():
    """Import the prebuilt extension (works without the reference checkout)."""
    so = OUT / f"{NAME}.so"
    if not so.exists():
        raise FileNotFoundError(f"{so} missing; run oracle/build_ref.py where the reference is available")
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(NAME, so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=pathlib.Path, default=DEFAULT_REFERENCE)
    print(build(ap.parse_args().reference))
