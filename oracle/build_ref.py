"""Build the reference project's own CUDA kernels from its sources into ``oracle/_ref/``.

TEST INFRASTRUCTURE ONLY (the checker, never the product).  Compiles, unmodified and where they
lie in the reference checkout, the three kernel/binding pairs the reference ships:

    src/attention.cu  + src/attention_binding.cpp -> oracle/_ref/custom_paged_attn/*.so
    src/fused_rope.cu + src/rope_binding.cpp      -> oracle/_ref/custom_rope/*.so
    src/fused_swiglu.cu + src/swiglu_binding.cpp  -> oracle/_ref/custom_swiglu/*.so

as PyTorch extensions for sm_100a (the reference builds with ``-arch=native``, setup.py:18).
The built modules travel with a copy of the repository to a machine with a B200 (``oracle/_ref``
is git-ignored, not excluded from copies); there ``load_ref(name)`` imports them so that
``tests/golden/make_kernel_golden.py`` can record the reference kernels' outputs.

    python oracle/build_ref.py --ref <reference checkout>
"""
from __future__ import annotations

import argparse
import glob
import importlib.util
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
# Where this recipe and tests/golden/make_golden.py look for the reference checkout when neither
# --ref nor TINY_INFRA_REF names one: the one place the checkout's location is written down.
_CHECKOUT = "/root/reference"


def reference_root(arg: str | None = None) -> str | None:
    """The reference checkout to read: ``arg``, else $TINY_INFRA_REF, else the build
    container's checkout if it exists there; None when there is none (e.g. on a GPU box)."""
    for cand in (arg, os.environ.get("TINY_INFRA_REF")):
        if cand:
            return cand
    return _CHECKOUT if os.path.isdir(os.path.join(_CHECKOUT, "src")) else None
MODULES = {
    "custom_paged_attn": ("src/attention.cu", "src/attention_binding.cpp"),
    "custom_rope": ("src/fused_rope.cu", "src/rope_binding.cpp"),
    "custom_swiglu": ("src/fused_swiglu.cu", "src/swiglu_binding.cpp"),
}


def build(ref_root: str, verbose: bool = False) -> list[str]:
    from torch.utils.cpp_extension import load

    built = []
    for name, srcs in MODULES.items():
        paths = [os.path.join(ref_root, s) for s in srcs]
        if not all(os.path.exists(p) for p in paths):
            raise FileNotFoundError(f"reference sources missing for {name}: {paths}")
        out = os.path.join(REF_OUT, name)
        os.makedirs(out, exist_ok=True)
        load(name=name, sources=paths, build_directory=out, verbose=verbose,
             extra_cflags=["-O3"],
             extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"])
        built.append(out)
    return built


def load_ref(name: str):
    """Import a module built by :func:`build` (works without the reference checkout)."""
    so = glob.glob(os.path.join(REF_OUT, name, f"{name}*.so"))
    if not so:
        raise FileNotFoundError(f"{name} not built under {REF_OUT}")
    import torch  # noqa: F401  (the extension links against libtorch)
    spec = importlib.util.spec_from_file_location(name, so[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=None, help="reference checkout (default: $TINY_INFRA_REF)")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    ref = reference_root(a.ref)
    if ref is None:
        ap.error("no reference checkout: pass --ref or set TINY_INFRA_REF")
    for p in build(ref, a.verbose):
        print("built", p)


if __name__ == "__main__":
    sys.exit(main())
