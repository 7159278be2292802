"""The C ABI header is plain C: a C99 program (-pedantic, warnings as errors) that includes
it compiles, links against the in-tree library and runs without a GPU."""
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

PROGRAM = r"""
#include "vibegemm_b200.h"
#include <stdio.h>
int main(void) {
    int out[20];
    int n = vg_b200_num_versions();
    int rc = vg_b200_plan(-1, 8192, 8192, 8192, 256, 256, 256, 0, 148, out);
    printf("%d %s %d %d\n", n, vg_b200_version_name(-1), rc, out[13]);
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="no C compiler")
def test_header_is_c99_and_links(vg, tmp_path):
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "abi"
    lib_dir = Path(vg.__file__).resolve().parent
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    f"-I{ROOT / 'include'}", str(src), "-o", str(exe), f"-L{lib_dir}",
                    "-lvibegemm_b200", f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()
    assert int(out[0]) == len(vg.versions())
    assert out[1:4] == ["VibeGEMM", "B200", "auto"]
    assert int(out[4]) == 0 and int(out[5]) == 3  # 8192^3 plans v3
