"""The library build when several processes find it stale at the same time
(one process per GPU under torchrun, each importing the package): exactly one
runs the compiler, the others wait for it and load its result, and no process
trips over another's temporary file.  Runs on CPU with a stand-in compiler in
a scratch directory; the real library is not touched."""
from __future__ import annotations

import os
import subprocess
import sys
import textwrap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "paged-speculative-engine_b200")

FAKE_NVCC = textwrap.dedent("""\
    #!{python}
    import sys, time
    out = sys.argv[sys.argv.index("-o") + 1]
    with open({count!r}, "a") as f:
        f.write("run\\n")
    time.sleep(1.0)  # long enough for the other processes to find the library stale too
    with open(out, "wb") as f:
        f.write(b"built")
""")

CHILD = textwrap.dedent("""\
    import sys
    sys.path.insert(0, {pkg!r})
    from pse import _build
    _build.CSRC = {csrc!r}
    _build.INCLUDE = {inc!r}
    _build.LIB = {lib!r}
    _build.SOURCES = ["k.cu"]
    print(_build.build())
""")


def test_concurrent_builds_compile_once(tmp_path):
    csrc, inc, libdir = tmp_path / "csrc", tmp_path / "include", tmp_path / "lib"
    for d in (csrc, inc, libdir):
        d.mkdir()
    (csrc / "k.cu").write_text("// stand-in source\n")
    (inc / "pse.h").write_text("// stand-in header\n")
    count = tmp_path / "compiler_runs"
    nvcc = tmp_path / "nvcc"
    nvcc.write_text(FAKE_NVCC.format(python=sys.executable, count=str(count)))
    nvcc.chmod(0o755)
    lib = libdir / "libpse.so"
    env = dict(os.environ, NVCC=str(nvcc))
    code = CHILD.format(pkg=PKG_DIR, csrc=str(csrc), inc=str(inc), lib=str(lib))
    procs = [subprocess.Popen([sys.executable, "-c", code], env=env, stdout=subprocess.PIPE,
                              stderr=subprocess.PIPE, text=True) for _ in range(3)]
    outs = [p.communicate(timeout=120) for p in procs]
    for p, (out, err) in zip(procs, outs):
        assert p.returncode == 0, err
        assert out.strip() == str(lib)
    assert lib.read_bytes() == b"built"
    assert count.read_text().count("run") == 1  # the waiting processes found it fresh
    assert not [f for f in os.listdir(libdir) if ".tmp" in f]


def test_stale_library_is_rebuilt(tmp_path):
    """A source newer than the library triggers one rebuild; a fresh library none."""
    csrc, inc, libdir = tmp_path / "csrc", tmp_path / "include", tmp_path / "lib"
    for d in (csrc, inc, libdir):
        d.mkdir()
    (csrc / "k.cu").write_text("// stand-in source\n")
    (inc / "pse.h").write_text("// stand-in header\n")
    count = tmp_path / "compiler_runs"
    nvcc = tmp_path / "nvcc"
    nvcc.write_text(FAKE_NVCC.format(python=sys.executable, count=str(count)).replace("time.sleep(1.0)", "pass"))
    nvcc.chmod(0o755)
    lib = libdir / "libpse.so"
    env = dict(os.environ, NVCC=str(nvcc))
    code = CHILD.format(pkg=PKG_DIR, csrc=str(csrc), inc=str(inc), lib=str(lib))
    run = lambda: subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert run().returncode == 0
    assert run().returncode == 0
    assert count.read_text().count("run") == 1
    t = os.path.getmtime(lib)
    os.utime(csrc / "k.cu", (t + 10, t + 10))
    assert run().returncode == 0
    assert count.read_text().count("run") == 2
