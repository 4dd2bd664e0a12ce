"""The device computes a Q8_0 block scale d = amax/127 with a multiply and one
FMA correction instead of a division (common.cuh div127_rn).  This checks, on
the CPU, that the formula equals IEEE division for all 2^31 non-negative
finite floats; it uses only correctly rounded multiply and FMA, so the same
holds bit for bit on the GPU."""
import os
import subprocess
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))


def test_div127_matches_ieee_division_exhaustively():
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "div127")
        subprocess.run(["gcc", "-O2", "-ffp-contract=off", "-mfma", "-o", exe,
                        os.path.join(HERE, "div127_exhaustive.c"), "-lm"], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
        assert out.returncode == 0 and out.stdout.strip() == "0", out.stdout
