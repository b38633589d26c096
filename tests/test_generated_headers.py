"""The TMEM load/store wrappers (blackwell_b200/csrc/tmem_io.cuh) are written
by gen_tmem_io.py; the committed header must be exactly what the generator
prints, so that an edit to one without the other is caught on CPU."""
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parents[1] / "blackwell_b200" / "csrc"


def test_tmem_io_header_matches_generator():
    out = subprocess.run([sys.executable, str(CSRC / "gen_tmem_io.py")], capture_output=True, text=True, check=True)
    assert out.stdout == (CSRC / "tmem_io.cuh").read_text()


def test_tmem_io_has_the_shapes_the_kernels_use():
    text = (CSRC / "tmem_io.cuh").read_text()
    for name in ("tmem_ld32", "tmem_ld64", "tmem_st32", "tmem_ld_16x256b_x16", "tmem_st_16x256b_x16",
                 "tmem_ld_16x256b_x8", "tmem_st_16x256b_x8", "tmem_st_16x128b_x16", "tmem_wait_st"):
        assert f"void {name}(" in text, name
