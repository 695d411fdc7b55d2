"""Build libts_attn.so in-tree with nvcc for sm_100a.

    python -m tensorsmith_b200._build        (from custom-ml-library_b200/)

Each ``csrc/*.cu`` is compiled to an object in parallel, then linked into
``tensorsmith_b200/lib/libts_attn.so`` (static CUDA runtime, no driver-library
link: the tensor-map encoder is fetched with cudaGetDriverEntryPoint).
"""

from __future__ import annotations

import concurrent.futures
import os
import re
import shutil
import subprocess
import sys
import time
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libts_attn.so"
INCLUDE = ROOT.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the B200 engine needs the CUDA toolkit to build")
    return found


def _source_digest() -> str:
    from ._lib import source_digest

    return source_digest()


DIGEST_STAMP = BUILD / "abi.digest"


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    digest = None
    if src.name == "abi.cu":
        # The library reports the digest of the sources it was built from (ts_attn_source_digest).
        digest = _source_digest()
        cmd.append(f'-DTS_SOURCE_DIGEST="{digest}"')
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    started = time.time()
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    # Stamp the object with the time its sources were read, so a source edited
    # while nvcc ran is newer than the object and gets rebuilt next time.
    os.utime(obj, (started, started))
    if digest is not None:
        DIGEST_STAMP.write_text(digest)
    return obj, res.stderr


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _library_digest() -> str | None:
    """Digest compiled into the library on disk (read in a child process, so this process never
    maps a library it may be about to replace)."""
    code = ("import ctypes,sys; f=ctypes.CDLL(sys.argv[1]).ts_attn_source_digest; "
            "f.restype=ctypes.c_char_p; print(f().decode())")
    res = subprocess.run([sys.executable, "-c", code, str(LIB)], capture_output=True, text=True)
    return res.stdout.strip() if res.returncode == 0 else None


def stale() -> bool:
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    if any(p.stat().st_mtime > built for p in deps):
        return True
    return _library_digest() != _source_digest()


_INCLUDE_RE = re.compile(r'^\s*#\s*include\s*"([^"]+)"', re.M)


def _local_deps(src: Path) -> set[Path]:
    """The file plus every quoted include reachable from it in csrc/ and include/."""
    seen: set[Path] = set()
    stack = [src]
    while stack:
        path = stack.pop()
        if path in seen or not path.exists():
            continue
        seen.add(path)
        for name in _INCLUDE_RE.findall(path.read_text(errors="replace")):
            for base in (path.parent, CSRC, INCLUDE):
                if (base / name).exists():
                    stack.append((base / name).resolve())
                    break
    return seen


def _object_stale(src: Path) -> bool:
    """An object is rebuilt when its source or a header it includes (transitively) is newer."""
    obj = BUILD / (src.stem + ".o")
    if not obj.exists():
        return True
    if src.name == "abi.cu" and (not DIGEST_STAMP.exists() or DIGEST_STAMP.read_text() != _source_digest()):
        return True
    built = obj.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _local_deps(src.resolve()))


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    if not force and not stale():
        return LIB
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    srcs = sources()
    todo = [s for s in srcs if force or verbose_ptxas or _object_stale(s)]
    jobs = jobs or max(1, min(len(todo), os.cpu_count() or 4))
    with concurrent.futures.ThreadPoolExecutor(jobs) as pool:
        results = list(pool.map(lambda s: _compile(s, verbose_ptxas), todo))
    if verbose_ptxas:
        for (_, log), src in zip(results, todo):
            sys.stderr.write(f"== {src.name}\n{log}")
    objects = [BUILD / (s.stem + ".o") for s in srcs]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(o) for o in objects]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv)
    print(path)
