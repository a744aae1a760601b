"""The package's device-side synthetic generator reproduces the reference generator (pinned oracle) exactly."""

import torch

from kimi_k3_goalbox_b200 import synthetic
from oracle import kimi_oracle as ko
from tests import gpu_helpers as gh
from tests.test_oracle_kat import tiny


def test_package_generator_matches_oracle():
    for case, seed in ((tiny(3), 21), (gh.small_case(2), 7), (tiny(1), 9)):
        want = ko.make_inputs(case, seed, "cpu")
        got = synthetic.make_inputs(case, seed, "cpu")
        assert set(got) == set(want)
        for k in want:
            assert got[k].dtype == want[k].dtype and torch.equal(got[k], want[k]), k
