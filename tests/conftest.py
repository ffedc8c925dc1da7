import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "xgboost-metal_b200"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=True)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
