"""Resource checks of the sm_100a kernels at compile time, without a GPU.

Every kernel source is compiled with the library's own flags plus
`-Xptxas -v` into a scratch directory.  Every kernel entry point must
report no spill stores or loads: a spill in a hot kernel is a silent
performance regression.  ptxas caps each kernel's registers at the budget
its launch bounds imply (threads x minimum CTAs per SM) and spills past it,
so the spill check also guards those budgets; registers per thread must
stay at or below 255.
"""
import os
import re
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(not shutil.which("nvcc") and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="nvcc not present")
def test_no_kernel_spills_registers(tmp_path):
    from hxinfer_b200 import build
    sources = sorted(f for f in os.listdir(build.CSRC) if f.endswith(".cu"))
    assert sources

    def compile_one(src):
        cmd = [build.nvcc()] + build.ARCH + build.NVCC_FLAGS + \
            ["-Xptxas", "-v", "-c", os.path.join(build.CSRC, src), "-o", str(tmp_path / (src + ".o"))]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, r.returncode, r.stdout + r.stderr

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(compile_one, sources))
    failed = [(s, out[-1500:]) for s, rc, out in results if rc != 0]
    assert not failed, failed

    spills, entries = [], 0
    for src, _, out in results:
        kernel = None
        for line in out.splitlines():
            m = re.search(r"Compiling entry function '(\S+)'", line)
            if m:
                kernel = m.group(1)
                entries += 1
                continue
            m = re.search(r"(\d+) bytes spill stores, (\d+) bytes spill loads", line)
            if m and kernel and (int(m.group(1)) or int(m.group(2))):
                spills.append((src, kernel[:80], line.strip()))
            m = re.search(r"Used (\d+) registers", line)
            if m and kernel:
                assert int(m.group(1)) <= 255, (src, kernel[:80], line)
    assert entries >= 10, "ptxas reported too few entry functions"
    assert not spills, spills
