"""enilnets_b200.hostmem: the NUMA binding around pinned-buffer allocation is
a no-op without NVML or a GPU and always restores the caller's CPU set."""
import os

from enilnets_b200 import hostmem


def test_local_to_restores_affinity():
    before = os.sched_getaffinity(0)
    with hostmem.local_to(0) as cpus:
        if cpus is None:
            assert os.sched_getaffinity(0) == before
        else:
            assert os.sched_getaffinity(0) == set(cpus)
    assert os.sched_getaffinity(0) == before


def test_local_to_restores_on_error():
    before = os.sched_getaffinity(0)
    try:
        with hostmem.local_to(0):
            raise RuntimeError("inside")
    except RuntimeError:
        pass
    assert os.sched_getaffinity(0) == before


def test_unknown_device_is_unbound():
    assert hostmem.gpu_local_cpus(10 ** 6) is None
