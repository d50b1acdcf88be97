"""The in-tree build: every source and header the library is compiled from triggers a rebuild
(an edit to a header that the dependency list missed once left a stale library in place)."""
import os

from invision_b200 import build


def test_every_source_is_a_build_dependency():
    csrc = os.path.join(os.path.dirname(build.__file__), "csrc")
    deps = set(build.deps())
    for f in os.listdir(csrc):
        if f.endswith((".cu", ".cuh", ".hpp", ".h")):
            assert os.path.join(csrc, f) in deps, f
    assert os.path.join(build.INCLUDE, "envgemm.h") in deps
