"""pytest set-up: import paths and the `gpu` marker.

`-m "not gpu"` runs everywhere (oracle, host logic, C-ABI loading);
`-m gpu` needs a B200 and calls the CUDA path through the C ABI.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
for p in (ROOT, ROOT / "lucciola-rs_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

# Attention outputs: max-abs error bound against the reference's algorithm
# (bf16 in, fp32 accumulate), as BASELINE.json's north_star states.
ATTN_ATOL = 2e-2


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU; calls the CUDA path")
