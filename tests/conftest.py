import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("oracle", os.path.join("vspec-engine_b200", "python")):
    path = os.path.join(ROOT, sub)
    if path not in sys.path:
        sys.path.insert(0, path)

# The reference's 3-bit runtime module switches int3/attention arithmetic
# through the environment (src/runtime/three_bit_runtime_modules.c:60-66); the
# oracle is pinned against the clean-environment ("raw") reference.
for var in ("VSPEC_3BIT_RUNTIME_MODULE", "VSPEC_FUSED_BITS"):
    os.environ.pop(var, None)

# The reference source tree (headers, Python modules) for the tests that read it:
# VSPEC_REFERENCE, else the build environment's default from __graft_entry__.
if not os.environ.get("VSPEC_REFERENCE"):
    sys.path.insert(0, ROOT)
    from __graft_entry__ import reference_tree  # noqa: E402
    if reference_tree():
        os.environ["VSPEC_REFERENCE"] = reference_tree()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def root():
    return ROOT
