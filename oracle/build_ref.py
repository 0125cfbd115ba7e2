"""Build recipe for oracle/_ref/ -- the reference's OWN CUDA kernels, compiled from their sources
where they lie in the reference checkout, for sm_100a.

TEST AND COMPARISON INFRASTRUCTURE ONLY.  Three torch extensions, each with the reference's own
compile flags (kernels/qwen35moe_gdn_prefill.py:49-61, kernels_optimized/flash_attention_2.py:45-62,
kernels_optimized/qwen35moe_gdn_prefill.py, same flag list) and the target architecture changed
from sm_89 to sm_100a:

  gdn_scalar  kernels/qwen35moe_gdn_prefill.cu            the fp32 recurrence (the maths definition);
                                                          run on a B200 it produced tests/golden/gdn_*.npz
  fa2_opt     kernels_optimized/flash_attention_2.cu      the reference's optimised FA2 (mma.sync)
  gdn_opt     kernels_optimized/qwen35moe_gdn_prefill.cu  the reference's optimised chunked GDN (wmma)

The two optimised kernels are timed beside this repository's kernels on the same B200 by
oracle/time_ref_kernels.py.  Nothing is copied out of the reference tree.

    python oracle/build_ref.py [--reference /path/to/reference] [--only gdn_scalar,fa2_opt,gdn_opt]
"""

from __future__ import annotations

import argparse
import importlib.util
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
DEFAULT_REFERENCE = pathlib.Path("/root/reference")

# target -> (source path inside the reference checkout, extension module name)
TARGETS = {
    "gdn_scalar": ("kernels/qwen35moe_gdn_prefill.cu", "ref_gdn_scalar"),
    "fa2_opt": ("kernels_optimized/flash_attention_2.cu", "ref_fa2_opt"),
    "gdn_opt": ("kernels_optimized/qwen35moe_gdn_prefill.cu", "ref_gdn_opt"),
}

_CFLAGS = ["-O3", "-std=c++17", "-w"]
_CUDA_CFLAGS = ["-O3", "-lineinfo", "-w", "--use_fast_math", "-std=c++17", "--expt-relaxed-constexpr",
                "--expt-extended-lambda", "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
                "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-gencode=arch=compute_100a,code=sm_100a"]


def so_path(target: str) -> pathlib.Path:
    return REF_OUT / target / f"{TARGETS[target][1]}.so"


def build(reference: pathlib.Path = DEFAULT_REFERENCE, only=None) -> list[pathlib.Path]:
    """Compile the selected targets (all by default); a target whose .so is newer than its source
    is left as it is."""
    from torch.utils.cpp_extension import load

    built = []
    for target in (only or TARGETS):
        rel, name = TARGETS[target]
        src = reference / rel
        if not src.exists():
            raise FileNotFoundError(src)
        out = so_path(target)
        if not (out.exists() and out.stat().st_mtime >= src.stat().st_mtime):
            out.parent.mkdir(parents=True, exist_ok=True)
            load(name=name, sources=[str(src)], build_directory=str(out.parent), verbose=False,
                 extra_cflags=_CFLAGS, extra_cuda_cflags=_CUDA_CFLAGS)
        built.append(out)
    return built


def load_built(target: str = "gdn_scalar"):
    """Import a prebuilt extension (works without the reference checkout)."""
    so = so_path(target)
    if not so.exists():
        raise FileNotFoundError(f"{so} missing; run oracle/build_ref.py where the reference is available")
    import torch  # noqa: F401  (the extension links against libtorch)

    spec = importlib.util.spec_from_file_location(TARGETS[target][1], so)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=pathlib.Path, default=DEFAULT_REFERENCE)
    ap.add_argument("--only", default="", help="comma-separated subset of " + ",".join(TARGETS))
    args = ap.parse_args()
    for p in build(args.reference, [t for t in args.only.split(",") if t] or None):
        print(p)
