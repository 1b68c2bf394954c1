"""The VMM helpers of the harness API on one GPU (include/vmm.cuh:12-38 of the
reference: vm_alloc = cuMemGetAllocationGranularity + cuMemCreate, vm_map =
cuMemAddressReserve + cuMemMap), through the C ABI: allocate, map, grant
access, write with a kernel, read back, unmap and free.  A second mapping of
the same physical allocation must show the bytes written through the first
(the slab's unicast and multicast views rely on exactly that)."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _check(L, rc, what):
    assert rc == 0, f"{what}: {L.agg_last_error().decode()}"


def test_vm_alloc_map_access_write_read_free(pkg, gpu):
    import torch

    L = pkg.lib()
    want = (3 << 20) + 4096  # not a multiple of the allocation granularity
    h = ctypes.c_uint64()
    size = ctypes.c_size_t()
    _check(L, L.agg_vm_alloc(ctypes.byref(h), ctypes.byref(size), want, 0), "agg_vm_alloc")
    assert size.value >= want and size.value % 4096 == 0, size.value
    devices = (ctypes.c_int * 1)(0)
    va = [ctypes.c_uint64(), ctypes.c_uint64()]
    try:
        for v in va:
            _check(L, L.agg_vm_map(ctypes.byref(v), h.value, size.value), "agg_vm_map")
            _check(L, L.agg_vm_set_access(v.value, size.value, devices, 1), "agg_vm_set_access")
        assert va[0].value != va[1].value
        n = size.value // 4
        first = pkg.agg.device_view(va[0].value, (n,), torch.int32)
        second = pkg.agg.device_view(va[1].value, (n,), torch.int32)
        pattern = torch.arange(n, dtype=torch.int32, device="cuda") * 7 + 3
        first.copy_(pattern)  # a copy kernel writes through the first mapping
        torch.cuda.synchronize()
        assert torch.equal(first.cpu(), pattern.cpu())
        assert torch.equal(second.cpu(), pattern.cpu())
        second.fill_(-1)  # and through the second
        torch.cuda.synchronize()
        assert int((first != -1).sum().item()) == 0
        del first, second
    finally:
        torch.cuda.synchronize()
        for v in va:
            if v.value:
                _check(L, L.agg_vm_unmap_free(v.value, size.value), "agg_vm_unmap_free")
        _check(L, L.agg_vm_release(h.value), "agg_vm_release")


def test_vm_set_access_rejects_empty_device_list(pkg):
    L = pkg.lib()
    assert L.agg_vm_set_access(0x10000, 4096, None, 0) == -1
