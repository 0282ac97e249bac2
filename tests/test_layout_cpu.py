"""include/dsv4_types.h must lay the reference's structs out exactly as the
reference's dsv4.h does (golden: tests/golden/layout_ref.txt, produced from
the reference header by tests/golden/make_layout.py). CPU only."""
import os
import subprocess
import tempfile

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_struct_layout_matches_reference():
    exe = os.path.join(tempfile.mkdtemp(), "layout_probe")
    subprocess.run(["/usr/bin/gcc", "-I" + os.path.join(REPO, "include"),
                    os.path.join(REPO, "tests", "golden", "layout_probe.c"), "-o", exe], check=True)
    mine = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
    golden = open(os.path.join(REPO, "tests", "golden", "layout_ref.txt")).read()
    assert mine == golden
