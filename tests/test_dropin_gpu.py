"""The drop-in check: the reference's own C callers, unchanged, on this library.

oracle/Makefile (target dropin, run by __graft_entry__.build() where the
reference sources exist) compiles the reference's examples/oneshot.c,
tests/test_generate.c and tests/test_threads.c from its own sources and with
its own include/cmol.h, and links them against libcmol_b200/lib/libcmol.so.
Their live sections load the model named "dropin.gguf" in the working
directory: here a synthetic one.  Each program must exit 0 with no FAIL line
(the reference's test harness prints PASS / FAIL per check and exits 1 on
any failure, tests/test_generate.c:476-477).
"""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DROPIN = os.path.join(ROOT, "oracle", "_ref", "dropin")


def _bin(name):
    p = os.path.join(DROPIN, name)
    if not os.path.exists(p):
        pytest.skip(f"{name} not built (needs the reference sources: make -C oracle dropin)")
    return p


@pytest.fixture(scope="module")
def workdir(tmp_path_factory):
    from libcmol_b200 import synth
    d = tmp_path_factory.mktemp("dropin")
    synth.write_gguf(str(d / "dropin.gguf"), synth.tiny_spec(synth.Q4_K, ctx=1024, eos=2))
    return str(d)


def _run(args, cwd):
    r = subprocess.run(args, cwd=cwd, capture_output=True, timeout=600)
    out = (r.stdout + r.stderr).decode("utf-8", "replace")   # generated text is arbitrary bytes
    return r.returncode, out


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["test_generate", "test_threads"])
def test_reference_tests_pass_on_libcmol(gpu, workdir, name):
    rc, out = _run([_bin(name)], workdir)
    print(out[-3000:])
    fails = [ln for ln in out.splitlines() if ln.strip().startswith("FAIL")]
    assert rc == 0 and not fails, (rc, fails)
    assert "Live tests skipped" not in out


@pytest.mark.gpu
def test_reference_oneshot_example(gpu, workdir):
    rc, out = _run([_bin("oneshot"), "dropin.gguf", "Hello there", "-t", "0", "-n", "8"], workdir)
    assert rc == 0, out
    assert out.strip(), "no text generated"
