"""The B200 family dropped into the reference's own tree and built by the reference's CMake.

A copy of the reference tree (VibeGEMM) gets the B200 family from vibegemm_b200.dropin:
new files, plus four additive edits of its registry, cuBLAS backend, main.cu and
CMakeLists.txt. Checked here: every original line survives, in order (nothing removed or
rewritten); the edits are what the installer documents; a second install changes nothing;
and `cmake -DTARGET_GPU=B200` configures and builds the reference's `VibeGEMM` driver with
the B200 backends registered in it. Runs where the reference tree and cmake are present
(VIBEGEMM_REFERENCE_DIR, else the build container's default location)."""
import os
import shutil
from pathlib import Path

import pytest

REFERENCE = Path(os.environ.get("VIBEGEMM_REFERENCE_DIR", "/root/reference"))

pytestmark = pytest.mark.skipif(not (REFERENCE / "CMakeLists.txt").is_file() or not shutil.which("cmake"),
                                reason="needs the reference tree and cmake")


def _is_subsequence(old: list[str], new: list[str]) -> bool:
    it = iter(new)
    return all(any(line == n for n in it) for line in old)


@pytest.fixture(scope="module")
def tree(tmp_path_factory):
    from vibegemm_b200 import dropin
    t = tmp_path_factory.mktemp("dropin") / "VibeGEMM"
    shutil.copytree(REFERENCE, t, ignore=shutil.ignore_patterns(".git", "build", "out", "results"))
    touched = dropin.install(t)
    return t, touched


def test_edits_are_additive(tree):
    from vibegemm_b200 import dropin
    t, touched = tree
    edited = {rel for rel, *_ in dropin.EDITS}
    assert edited == {"include/registry.cuh", "csrc/cublas_backends.cu", "main.cu", "CMakeLists.txt"}
    for rel in edited:
        old = (REFERENCE / rel).read_text().split("\n")
        new = (t / rel).read_text().split("\n")
        assert _is_subsequence(old, new), rel
        added = len(new) - len(old)
        want = sum(len(lines) for r, _, _, lines in dropin.EDITS if r == rel)
        assert added == want, (rel, added, want)
    for rel, _src in dropin.NEW_FILES:
        assert (t / rel).is_file() and not (REFERENCE / rel).exists(), rel
    # The reference's headers the engine and the registrations compile against are its own.
    for rel in ("include/backend.cuh", "include/engine.cuh", "include/utils.cuh"):
        assert (t / rel).read_bytes() == (REFERENCE / rel).read_bytes(), rel
    assert "REGISTER_B200_KERNEL(dn, BC)  _KREG_IMPL(3, dn, BC, __COUNTER__)" in (t / "include/registry.cuh").read_text()


def test_second_install_is_a_no_op(tree):
    from vibegemm_b200 import dropin
    t, _ = tree
    before = {p: p.read_bytes() for p in t.rglob("*") if p.is_file()}
    dropin.install(t)
    after = {p: p.read_bytes() for p in t.rglob("*") if p.is_file()}
    assert before == after


def test_install_refuses_a_tree_without_its_anchors(tmp_path):
    from vibegemm_b200 import dropin
    t = tmp_path / "other"
    shutil.copytree(REFERENCE, t, ignore=shutil.ignore_patterns(".git", "build", "out", "results"))
    cm = t / "CMakeLists.txt"
    cm.write_text(cm.read_text().replace('elseif(TARGET_GPU STREQUAL "A100")', 'elseif(TARGET_GPU MATCHES "A100")'))
    with pytest.raises(dropin.DropinError):
        dropin.install(t)


def test_reference_cmake_builds_the_b200_family(tree):
    from vibegemm_b200 import dropin
    t, _ = tree
    exe = dropin.build(t, jobs=os.cpu_count() or 8)
    data = exe.read_bytes()
    for v in [f"v{i}" for i in range(13)] + ["auto"]:
        assert f"VibeGEMM B200 {v}".encode() in data
    # the reference's own cuBLAS backend, compiled with the HAS_B200 arm, is in it too
    assert b"cuBLAS" in data and b"results/perf_b200.txt" in data
