"""CPU: host model of the kernels' scalar algorithms (exact_math.cuh):
the table-driven exp against glibc expf, and the parallel binade-chain
engine against the serial fp32 loop it must reproduce bit for bit."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))


def test_exp_and_chain_model(tmp_path):
    exe = tmp_path / "exact_math_model"
    subprocess.run(["g++", "-O2", "-std=c++17", "-o", str(exe), os.path.join(HERE, "model", "exact_math_model.cpp"),
                    "-lm"], check=True)
    out = subprocess.run([str(exe), "97"], capture_output=True, text=True)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
