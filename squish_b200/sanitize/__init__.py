"""Sanitizer builds of the host C++ libraries (the code that parses untrusted input: JSON
schemas from HTTP requests in grammar.cpp, checkpoint bytes in entropy.cpp, arrays of any
shape in cpu_ref.cpp, token streams in host_utils.cpp).

``build()`` compiles those sources into the module ``_C_host_asan`` with AddressSanitizer and
UndefinedBehaviorSanitizer (``-fsanitize=address,undefined``, no recovery from UB, frame
pointers kept) under ``build/asan`` in the repository, rebuilding only when a source
changed. ``run(script)`` executes Python code in a child process with the sanitizer runtime
preloaded (CPython and libtorch are not instrumented; leak checking is off because the
interpreter does not free everything at exit); any sanitizer report fails the child.

    python -c "from squish_b200 import sanitize; print(sanitize.run('import _C_host_asan'))"
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
CSRC = os.path.join(ROOT, "squish_b200", "csrc")
BUILD = os.path.join(ROOT, "build", "asan")
SOURCES = ["host_module.cpp", "cpu_ref.cpp", "entropy.cpp", "host_utils.cpp", "grammar.cpp", "quant_research.cpp",
           "kv_research.cpp", "recurrent.cpp"]
FLAGS = ["-O1", "-g", "-std=c++17", "-fsanitize=address,undefined", "-fno-omit-frame-pointer",
         "-fno-sanitize-recover=undefined", "-fno-sanitize=vptr"]


def compiler() -> str:
    """A g++ that ships the sanitizer runtimes (the first on PATH whose libasan resolves)."""
    for cxx in (os.environ.get("SQ_SANITIZE_CXX"), "g++", "/usr/bin/g++"):
        if not cxx:
            continue
        try:
            out = subprocess.run([cxx, "-print-file-name=libasan.so"], capture_output=True, text=True, check=True)
        except (OSError, subprocess.CalledProcessError):
            continue
        if os.path.isabs(out.stdout.strip()) and os.path.exists(out.stdout.strip()):
            return cxx
    raise RuntimeError("no g++ with an AddressSanitizer runtime (libasan) was found")


def runtime() -> str:
    """Path of the AddressSanitizer runtime of the compiler that builds the module."""
    out = subprocess.run([compiler(), "-print-file-name=libasan.so"], capture_output=True, text=True, check=True)
    return out.stdout.strip()


def _build_here(verbose: bool = False) -> None:
    from torch.utils.cpp_extension import load

    os.makedirs(BUILD, exist_ok=True)
    os.environ["CXX"] = compiler()  # torch.utils.cpp_extension compiles and links with $CXX
    load(name="_C_host_asan", sources=[os.path.join(CSRC, s) for s in SOURCES], extra_cflags=FLAGS,
         extra_ldflags=["-fsanitize=address,undefined"], build_directory=BUILD, verbose=verbose,
         with_cuda=False, is_python_module=True)


def build(verbose: bool = False, timeout: float = 900.0) -> str:
    """Compile (if a source changed) and return the directory holding ``_C_host_asan*.so``.
    The build runs in a child with the sanitizer runtime preloaded, because compiling ends
    with importing the module."""
    r = run(f"from squish_b200 import sanitize; sanitize._build_here({bool(verbose)})", timeout=timeout,
            build_first=False)
    if r.returncode != 0:
        raise RuntimeError(f"sanitizer build failed ({r.returncode}):\n{r.stdout[-2000:]}\n{r.stderr[-4000:]}")
    return BUILD


def run(code: str, timeout: float = 600.0, build_first: bool = True) -> subprocess.CompletedProcess:
    """Run ``code`` in a fresh interpreter with the sanitizer runtime preloaded and the
    sanitized module importable as ``_C_host_asan``."""
    if build_first:
        build()
    env = dict(os.environ)
    # the C++ runtime must be loaded when the sanitizer starts, or its exception interceptor
    # finds no __cxa_throw to forward to (CPython itself does not link libstdc++)
    cxx_rt = subprocess.run([compiler(), "-print-file-name=libstdc++.so.6"], capture_output=True, text=True,
                            check=True).stdout.strip()
    env["LD_PRELOAD"] = " ".join([runtime(), cxx_rt])
    env["ASAN_OPTIONS"] = "detect_leaks=0:abort_on_error=0:halt_on_error=1:exitcode=86"
    env["UBSAN_OPTIONS"] = "halt_on_error=1:print_stacktrace=1:exitcode=87"
    env["PYTHONPATH"] = os.pathsep.join([BUILD, ROOT, env.get("PYTHONPATH", "")])
    env["CXX"] = compiler()
    prelude = "import torch\n"  # libtorch first: the module links against it
    return subprocess.run([sys.executable, "-c", prelude + code], env=env, capture_output=True, text=True,
                          timeout=timeout)


__all__ = ["build", "run", "runtime"]
