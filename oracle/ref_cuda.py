"""The reference's own CUDA decode kernel, built for sm_100a (TEST INFRASTRUCTURE).

kvssd ships `csrc/fused_decode.cu` + `csrc/bindings.cpp` (the `kvssd._C` extension,
`setup.py:12-22`: nvcc -O3 --use_fast_math -lineinfo). `build()` compiles those two files where
they lie in the reference checkout -- nothing is copied -- into `oracle/_ref/` (git-ignored; the
built module travels to the GPU box with the rest of the tree). `load()` imports the built
module without the sources. Only tests use it: as a second parity pin (our kernels against the
reference's kernel on the same inputs) and as the reference GPU timing beside ours.

The reference checkout is found through $KVSSD_REFERENCE, else a `reference` directory next to
this repository.
"""

from __future__ import annotations

import importlib.util
import os
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "kvssd_ref_cuda"


def reference_root() -> Path:
    env = os.environ.get("KVSSD_REFERENCE")
    return Path(env) if env else HERE.parent.parent / "reference"


def sources() -> list[Path]:
    root = reference_root()
    return [root / "csrc" / "bindings.cpp", root / "csrc" / "fused_decode.cu"]


def built_module() -> Path | None:
    found = sorted(OUT.glob(f"{NAME}*.so"))
    return found[0] if found else None


def build(verbose: bool = False) -> Path | None:
    """Compiles the reference extension into oracle/_ref/ (None when the sources are absent)."""
    srcs = sources()
    if not all(s.exists() for s in srcs):
        return None
    from torch.utils import cpp_extension

    build_dir = OUT / "build"
    build_dir.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    cpp_extension.load(
        name=NAME,
        sources=[str(s) for s in srcs],
        build_directory=str(build_dir),
        extra_cflags=["-O3"],
        extra_cuda_cflags=["-O3", "--use_fast_math", "-lineinfo",
                           "-gencode", "arch=compute_100a,code=sm_100a"],
        verbose=verbose,
        is_python_module=True,
    )
    built = sorted(build_dir.glob(f"{NAME}*.so"))
    if not built:
        return None
    target = OUT / built[0].name
    target.write_bytes(built[0].read_bytes())
    return target


def load():
    """The built reference module (exposing `fused_decode`), or None if it was not built."""
    path = built_module()
    if path is None:
        return None
    import torch  # noqa: F401  (the extension links against torch's libraries)

    spec = importlib.util.spec_from_file_location(NAME, path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module
