"""Regenerate the golden fixtures of tests/golden/ from the reference (run in a
container where the reference checkout is available; the fixtures are
committed, so the tests themselves never need the reference).

  python tests/golden/make_golden.py /path/to/ponni-reference

pytorch_resnet.ponni: the reference's own fixture generator
unit/pytorch_resnet/generate_pytorch_resnet_data.py (TinyResNet 12->5 SiLU x4
residual ->4, seed 9012, one test sample; torch computes test.output), run
unmodified with the reference's generator package on PYTHONPATH.

projection_skip.ponni: the reference's unit/projection_skip/
generate_projection_skip_data.py (main and skip Linear 2->3 with fixed
weights and the expected outputs of its test), run the same way.
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("PONNI_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    env = dict(os.environ, PYTHONPATH=os.path.join(ref, "src", "generator"), CUDA_VISIBLE_DEVICES="")
    subprocess.run([sys.executable, os.path.join(ref, "unit", "pytorch_resnet", "generate_pytorch_resnet_data.py"),
                    os.path.join(HERE, "pytorch_resnet.ponni")], check=True, env=env)
    subprocess.run([sys.executable, os.path.join(ref, "unit", "projection_skip", "generate_projection_skip_data.py"),
                    os.path.join(HERE, "projection_skip.ponni")], check=True, env=env)


if __name__ == "__main__":
    main()
