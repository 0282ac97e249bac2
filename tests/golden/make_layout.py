"""Record the reference's struct layout (sizeof/offsetof of its model-level
types) into tests/golden/layout_ref.txt by compiling layout_probe.c against
the reference's include/dsv4/dsv4.h. Needs the reference checkout."""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
# the reference checkout: argument, REF_DIR, else `reference` beside the repository
REF = (sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_DIR")
       or os.path.join(os.path.dirname(os.path.dirname(os.path.dirname(HERE))), "reference"))
exe = "/tmp/layout_probe_ref"
subprocess.run(["/usr/bin/gcc", "-DUSE_REF", "-I" + os.path.join(REF, "include", "dsv4"),
                os.path.join(HERE, "layout_probe.c"), "-o", exe], check=True)
out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout
open(os.path.join(HERE, "layout_ref.txt"), "w").write(out)
print(out)
