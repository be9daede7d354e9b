"""The package's smoke entry (one small QCAU forward, one decode layer step,
the KV build's FP8 stage and the indexer's top-k, each against the oracle),
run as a test so that a change that breaks it fails the GPU suite."""
import pytest


@pytest.mark.gpu
def test_smoke_entry():
    import __graft_entry__

    __graft_entry__.smoke()
