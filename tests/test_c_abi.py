"""The drop-in boundary from C: tests/c/vit_block_abi.c is the reference's
vit_block (sam3_model.c:981-1028) written against include/sam3_cuda.h with
the operator macros of INTEGRATION.md section 3 pasted unchanged.

  * (CPU) the macro block in INTEGRATION.md is the one in the C file, and
    the file compiles with gcc -std=gnu11 -Wall -Werror and links against
    libsam3cuda.so (no GPU needed to build);
  * (GPU) the program's output for a windowed and a global block matches the
    oracle's vit_block on the same seeded weights (cosine >= 0.999 on the
    block's update, the bound of the encoder tests).
"""
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c", "vit_block_abi.c")
LIBDIR = os.path.join(ROOT, "i.sam3.opencl_b200")


def _build(tmp_path):
    if not os.path.exists(os.path.join(LIBDIR, "libsam3cuda.so")):
        pytest.skip("libsam3cuda.so not built")
    exe = str(tmp_path / "vit_block_abi")
    subprocess.run(["gcc", "-std=gnu11", "-O2", "-Wall", "-Wextra", "-Werror",
                    "-I" + os.path.join(ROOT, "include"), SRC, "-o", exe,
                    "-L" + LIBDIR, "-lsam3cuda", "-Wl,-rpath," + LIBDIR, "-lm"],
                   check=True, capture_output=True, text=True)
    return exe


def test_integration_macros_are_the_ones_compiled():
    doc = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    sec = doc[doc.index("## 3."):doc.index("## 4.")]
    block = re.search(r"```c\n(.*?)```", sec, re.S).group(1)
    src = open(SRC).read()
    assert block.strip() in src


def test_c_consumer_compiles_against_header(tmp_path):
    assert os.path.exists(_build(tmp_path))


@pytest.mark.gpu
@pytest.mark.parametrize("kind", [0, 1])
def test_c_vit_block_vs_oracle(tmp_path, ob, kind):
    exe = _build(tmp_path)
    seed = 31
    out = str(tmp_path / "x.f32")
    r = subprocess.run([exe, out, str(seed), str(kind)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    got = np.fromfile(out, np.float32).reshape(5184, 1024)
    x0 = ob.normal(seed, 99, (5184, 1024))
    w = ob.TrunkWeights(seed, depth=2, global_blocks=(1,))
    want = x0.copy()
    ob.encode_trunk(w, None, kind, kind + 1, x=want)
    a, b = (got - x0).astype(np.float64).ravel(), (want - x0).astype(np.float64).ravel()
    cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
    assert cos >= 0.999, cos
