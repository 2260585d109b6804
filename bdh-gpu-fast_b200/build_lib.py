"""Build recipe for libbdh_sm100.so (the C-ABI library of the sm_100a kernels) and for
bdh_sm100_ext.so (the PyTorch extension that binds it under the reference module's names).

Plain nvcc, no torch extension machinery: every .cu / .cpp under csrc/ is compiled for
sm_100a (-gencode arch=compute_100a,code=sm_100a) with -lineinfo, linked with a static CUDA
runtime into one shared object next to this file. Rebuilds only when a source or header is
newer than the library, and then only the objects whose source (or any header) changed; the
sources compile in parallel. Run as a script or call build().
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "libbdh_sm100.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile csrc/ into libbdh_sm100.so (in place). Returns the library path."""
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    headers = [p for p in _deps() if p.suffix in (".h", ".cuh")]
    newest_header = max((p.stat().st_mtime for p in headers), default=0.0)

    def compile_one(src: Path):
        obj = BUILD / (src.name + ".o")
        log = BUILD / (src.name + ".log")
        if (not force and obj.exists() and log.exists()
                and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header)):
            return str(obj), log.read_text(), 0
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        text = f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}"
        if r.returncode == 0:
            log.write_text(text)
        return str(obj), text, r.returncode

    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as pool:
        results = list(pool.map(compile_one, _sources()))
    objs = [o for o, _, _ in results]
    logs = [t for _, t, _ in results]
    failed = [Path(o).name for o, _, rc in results if rc != 0]
    if failed:
        sys.stderr.write("\n".join(logs))
        raise RuntimeError(f"nvcc failed on {', '.join(failed)}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-Xlinker", f"-soname={LIB.name}", "-o",
           str(tmp), *objs]
    r = subprocess.run(cmd, capture_output=True, text=True)
    logs.append(f"$ {' '.join(cmd)}\n{r.stdout}{r.stderr}")
    if r.returncode != 0:
        sys.stderr.write("\n".join(logs))
        raise RuntimeError("nvcc link failed")
    os.replace(tmp, LIB)
    (BUILD / "build.log").write_text("\n".join(logs))
    if verbose:
        print("\n".join(logs))
    return LIB


EXT_SRC = HERE / "ext" / "bdh_sm100_ext.cpp"
EXT_BUILD = BUILD / "ext"
EXT = HERE / "bdh_sm100_ext.so"


def ext_up_to_date() -> bool:
    if not EXT.exists():
        return False
    t = EXT.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in (EXT_SRC, *sorted(INCLUDE.glob("*.h"))))


def build_ext(force: bool = False, verbose: bool = False) -> Path:
    """Compile ext/bdh_sm100_ext.cpp (the PyTorch extension over the C-ABI, linked against
    libbdh_sm100.so through an $ORIGIN run path) into bdh_sm100_ext.so next to this file."""
    if not force and ext_up_to_date():
        return EXT
    if not LIB.exists():
        build()
    from torch.utils import cpp_extension

    EXT_BUILD.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name="bdh_sm100_ext", sources=[str(EXT_SRC)], extra_include_paths=[str(INCLUDE)],
        extra_cflags=["-O2"],
        # "$ORIGIN" escaped for ninja ($$) and the shell (\\$): the run path stays literal
        extra_ldflags=[f"-L{HERE}", "-lbdh_sm100", "-Wl,-rpath,\\$$ORIGIN:\\$$ORIGIN/../.."],
        build_directory=str(EXT_BUILD), with_cuda=True, verbose=verbose, is_python_module=True)
    built = EXT_BUILD / "bdh_sm100_ext.so"
    tmp = EXT.with_suffix(".so.tmp")
    shutil.copy2(built, tmp)
    os.replace(tmp, EXT)
    return EXT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIB)
    if "--ext" in sys.argv:
        print(build_ext(force="--force" in sys.argv, verbose="-v" in sys.argv))
