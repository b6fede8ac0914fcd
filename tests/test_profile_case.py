"""The profiling case runner parses its arguments and needs a GPU to run."""

from __future__ import annotations

import pytest
import torch

from gpumode_qr_b200 import profile_case


def test_argument_checks():
    with pytest.raises(SystemExit):
        profile_case.main(["unknown", "1", "2"])


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU exit")
def test_exits_without_a_gpu():
    assert profile_case.main(["gram", "2", "64", "64"]) == 2
