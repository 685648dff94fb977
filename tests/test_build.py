"""Properties of the built extension that need no GPU."""
import os
import subprocess

import pytest

from dtrain_b200.ops import _ext


@pytest.mark.skipif(not _ext.available(), reason="extension not built")
def test_extension_uses_the_shared_cxx_runtime():
    """A static libstdc++ copy inside the extension mixes with the process's shared
    one and turns the first numeric error message into a SIGSEGV; the build must
    link libstdc++.so dynamically."""
    out = subprocess.run(["readelf", "-d", _ext.built_path()], capture_output=True, text=True, check=True).stdout
    needed = [l for l in out.splitlines() if "(NEEDED)" in l]
    assert any("libstdc++.so" in l for l in needed), needed


def test_shared_libstdcxx_link_input_is_found():
    import torch  # noqa: F401  (loads the C++ runtime into this process)
    inputs = _ext._shared_libstdcxx()
    assert inputs and ("libstdc++.so" in os.path.basename(inputs[0]) or inputs[0].startswith("-l:"))


def test_every_native_source_is_built():
    """build() compiles every .cu / .cpp file of csrc/ (a new kernel file must not be left out)."""
    on_disk = sorted(f for f in os.listdir(_ext.SRC_DIR) if f.endswith((".cu", ".cpp")))
    assert sorted(_ext.SOURCES) == on_disk
    assert "arch=compute_100a,code=sm_100a" in " ".join(_ext.CUDA_FLAGS)
