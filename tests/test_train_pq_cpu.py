"""TrainPQ's option and input checks (PQOptions.Validate, pq.go:66-84; the
dimension and chunk checks and validateTrainingVectors of TrainPQ,
pq.go:118-136): xvec_gpu_pq_train rejects these on the host, before any
device call, so they run without a GPU."""
import numpy as np
import pytest

from oracle.oracle import COSINE, IP, L2, MIPSL2


@pytest.fixture(scope="module")
def xb():
    import xvec_b200
    return xvec_b200


@pytest.mark.parametrize("kwargs", [{"metric": COSINE}, {"metric": MIPSL2}, {"chunks": 9},
                                    {"chunks": -1}, {"max_train_samples": 0},
                                    {"max_iterations": 0}])
def test_invalid_options(xb, kwargs):
    x = np.ones((50, 8), np.float32)
    args = {"metric": L2, "chunks": 2, "max_train_samples": 100, "max_iterations": 2}
    args.update(kwargs)
    with pytest.raises(xb.XvecGPUError) as e:
        xb.pq_train(args["metric"], x, args["chunks"], args["max_train_samples"],
                    args["max_iterations"])
    assert e.value.status == xb.INVALID_ARGUMENT


def test_empty_and_non_finite(xb):
    with pytest.raises(xb.XvecGPUError) as e:
        xb.pq_train(L2, np.zeros((0, 8), np.float32), 2)
    assert e.value.status == xb.INVALID_ARGUMENT
    bad = np.ones((50, 8), np.float32)
    bad[49, 3] = np.nan          # past the training sample: still validated
    with pytest.raises(xb.XvecGPUError) as e:
        xb.pq_train(IP, bad, 2, 10, 2)
    assert e.value.status == xb.NON_FINITE
    assert "training vector 49" in str(e.value)


def test_oracle_agrees_on_invalid_options(oracle):
    x = np.ones((50, 8), np.float32)
    assert oracle.pq_train(COSINE, x, 2)[0] != 0
    assert oracle.pq_train(L2, x, 9)[0] != 0
    assert oracle.pq_train(L2, x, 2, max_train_samples=0)[0] != 0
    assert oracle.pq_train(L2, x, 2, max_iterations=0)[0] != 0
