import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HERE = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, HERE):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built extension")


# GPU tests fail loudly (they are not skipped) when no GPU is visible: the driver
# runs them on a B200 with `-m gpu`, and a silent skip would hide a broken build.


@pytest.fixture(scope="session")
def corpus(tmp_path_factory):
    """A small offline text corpus: pseudo-words built from a fixed syllable set."""
    rng = np.random.default_rng(7)
    syllables = ["ar", "be", "ci", "do", "el", "fa", "gu", "ho", "is", "ju", "ka", "lo"]
    words = ["".join(rng.choice(syllables, int(rng.integers(1, 4)))) for _ in range(48)]
    lines = [" ".join(rng.choice(words, 12)) for _ in range(400)]
    path = tmp_path_factory.mktemp("corpus") / "text.txt"
    path.write_text("\n".join(lines) + "\n")
    return str(path)
