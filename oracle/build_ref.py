"""Recipe: compile the reference's own CPU tril-attention extension into oracle/_ref/ — TEST
INFRASTRUCTURE ONLY (checker and timed CPU baseline; never part of the product path).

Sources are compiled where they lie in the read-only reference checkout
(``csrc/tril_attn_cpu.cpp`` + ``csrc/tril_attn_bind.cpp``, CPU only, no ``WITH_CUDA``), with
g++ through ``torch.utils.cpp_extension.load`` (the same compiler driver the reference's
``setup.py`` CppExtension uses; the reference's own build system is not run). Build files and
the resulting ``bdh_ref_ext*.so`` go to ``oracle/_ref/`` (git-ignored; it travels to the GPU
host with the working tree, where ``load()`` imports the prebuilt module without the sources).

Usage: ``python oracle/build_ref.py [/path/to/reference]``; without an argument the checkout is
``$BDH_REFERENCE`` or the ``reference_path`` of ``BASELINE.json``.
"""

from __future__ import annotations

import glob
import importlib.machinery
import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
NAME = "bdh_ref_ext"


def reference_root() -> Path | None:
    """Where the reference checkout is: ``$BDH_REFERENCE``, else the ``reference_path`` recorded
    in the repository's ``BASELINE.json``; None when neither names an existing directory."""
    env = os.environ.get("BDH_REFERENCE")
    cands = [Path(env)] if env else []
    try:
        import json

        rec = json.loads((HERE.parent / "BASELINE.json").read_text())
        if rec.get("reference_path"):
            cands.append(Path(rec["reference_path"]))
    except (OSError, ValueError):
        pass
    for c in cands:
        if c.is_dir():
            return c
    return None


def built_path() -> Path | None:
    hits = sorted(glob.glob(str(REF_OUT / f"{NAME}*.so")))
    return Path(hits[0]) if hits else None


def build(reference: Path | None = None, verbose: bool = False) -> Path:
    """Compile the reference CPU extension (if the reference sources are present)."""
    if reference is None:
        reference = reference_root()
    if reference is None:
        raise FileNotFoundError("no reference checkout: set BDH_REFERENCE")
    src = [reference / "csrc" / "tril_attn_cpu.cpp", reference / "csrc" / "tril_attn_bind.cpp"]
    if not all(p.exists() for p in src):
        raise FileNotFoundError(f"reference sources not found under {reference}/csrc")
    REF_OUT.mkdir(parents=True, exist_ok=True)
    from torch.utils.cpp_extension import load

    load(
        name=NAME,
        sources=[str(p) for p in src],
        extra_cflags=["-O3", "-std=c++20"],
        extra_include_paths=[str(reference / "csrc")],
        build_directory=str(REF_OUT),
        verbose=verbose,
        with_cuda=False,
    )
    p = built_path()
    if p is None:
        raise RuntimeError("reference extension did not produce a shared object")
    return p


def load_module():
    """Import the prebuilt reference extension from oracle/_ref (no compilation)."""
    import torch  # noqa: F401  (the extension links against libtorch)

    p = built_path()
    if p is None:
        raise ImportError("oracle/_ref has no built reference extension; run oracle/build_ref.py")
    if NAME in sys.modules:
        return sys.modules[NAME]
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(p))
    spec = importlib.util.spec_from_file_location(NAME, str(p), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[NAME] = mod
    return mod


if __name__ == "__main__":
    ref = Path(sys.argv[1]) if len(sys.argv) > 1 and sys.argv[1] != "-v" else None
    print(build(ref, verbose="-v" in sys.argv))
