"""The reference's own test files, unchanged, against this repository's module (GPU).

haowen-han/tma-depthwise-conv ships two test files for the operator:
``tests/test_dwconv.py`` (10 shapes, ``dwconv_v0`` and ``dwconv_ws`` at
n_stage 2/3/4 against ``ref_dwconv``) and ``tests/test_ws_time.py`` (the
``dwconv_ws_probe`` stall report on four shapes).  ``oracle/build_ref.py``
copies them, byte for byte, into the git-ignored ``oracle/_ref/tests/`` when a
reference checkout is named at build time, so they are available where no
checkout exists.  Each runs here in a child process that imports this
repository's ``tma_dwconv`` first: the files' own ``import tma_dwconv`` then
binds to it, which the child asserts before handing the file to pytest.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "tma-depthwise-conv_b200")
STAGED = os.path.join(REPO, "oracle", "_ref", "tests")

CHILD = r"""
import os, sys
pkg, path = sys.argv[1], sys.argv[2]
sys.path.insert(0, pkg)
import tma_dwconv
assert os.path.dirname(os.path.abspath(tma_dwconv.__file__)) == os.path.abspath(pkg), tma_dwconv.__file__
print("tma_dwconv from", tma_dwconv.__file__, flush=True)
import pytest
sys.exit(pytest.main([path, "-q", "-s", "-p", "no:cacheprovider", "-c", os.devnull,
                      "--rootdir", os.path.dirname(path)]))
"""


@pytest.mark.parametrize("name", ["test_dwconv.py", "test_ws_time.py"])
def test_reference_test_file_passes_against_this_module(name):
    path = os.path.join(STAGED, name)
    if not os.path.exists(path):
        pytest.skip("the reference's test files are not staged (oracle/build_ref.py with "
                    "TDC_REFERENCE_DIR)")
    r = subprocess.run([sys.executable, "-c", CHILD, PKG, path], capture_output=True, text=True,
                       timeout=1200, cwd=STAGED)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert f"tma_dwconv from {os.path.join(PKG, 'tma_dwconv.py')}" in out
    assert " passed" in out and " failed" not in out, out[-2000:]
