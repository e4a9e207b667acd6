"""The gather's no-allocation C entry point (``ft_p2p_gather_noalloc``) against the regular
entry point with a caller-owned counter buffer, on one GPU.

Two "ranks" are emulated on one device: two heaps, the peer's flag for the slot set before the
launch (so the gather never waits on another launch), rank 0 pulling rank 1's stripe. The
entry point is called through its exported C symbol, twice in a row, and must copy exactly
the bytes the regular entry point copies. Collected last so it also runs after every other
GPU test in the same process."""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("needs a CUDA device", allow_module_level=True)

from flextensor_b200.ops import native  # noqa: E402

DEV = torch.device("cuda", 0)
WORLD, N_SLOTS, SLOT = 2, 3, 1
SLOT_OFF = 4096
TOTAL = 3 * 1024 * 1024 + 512          # packed block size (multiple of 16)
STRIPE = ((TOTAL + WORLD - 1) // WORLD + 255) // 256 * 256


def _fn():
    lib = ctypes.CDLL(native.lib().__file__)
    f = lib.ft_p2p_gather_noalloc
    P = ctypes.POINTER(ctypes.c_uint64)
    u64, i32 = ctypes.c_uint64, ctypes.c_int
    f.argtypes = [P, P, P, i32, i32, i32, i32, u64, u64, u64, u64, i32, ctypes.c_void_p]
    f.restype = ctypes.c_int
    return f


class Ranks:
    """Heaps and flag/ack arrays of two emulated ranks; rank 0's heap is the destination."""

    def __init__(self, src_heap: torch.Tensor):
        self.heap0 = torch.zeros(SLOT_OFF + TOTAL, dtype=torch.uint8, device=DEV)
        self.heap1 = src_heap
        self.flags = [torch.zeros(WORLD * N_SLOTS, dtype=torch.int64, device=DEV) for _ in range(WORLD)]
        self.acks = [torch.zeros(WORLD * N_SLOTS, dtype=torch.int64, device=DEV) for _ in range(WORLD)]

    def ptrs(self):
        return ([self.heap0.data_ptr(), self.heap1.data_ptr()], [f.data_ptr() for f in self.flags],
                [a.data_ptr() for a in self.acks])

    def publish_peer(self, epoch):
        self.flags[0][1 * N_SLOTS + SLOT] = epoch  # rank 1 published its stripe of SLOT


def _run_pair(epoch, ctas):
    g = torch.Generator(device=DEV).manual_seed(epoch)
    src = torch.randint(0, 256, (SLOT_OFF + TOTAL,), dtype=torch.uint8, device=DEV, generator=g)
    a, b = Ranks(src), Ranks(src)
    a.publish_peer(epoch)
    b.publish_peer(epoch)
    h, f, k = a.ptrs()
    counters = torch.zeros(N_SLOTS, dtype=torch.int32, device=DEV)
    native.lib().p2p_gather_raw(h, f, k, 0, N_SLOTS, SLOT, epoch, SLOT_OFF, STRIPE, TOTAL, counters, ctas)

    h, f, k = b.ptrs()
    arr = lambda xs: (ctypes.c_uint64 * WORLD)(*xs)  # noqa: E731
    rc = _fn()(arr(h), arr(f), arr(k), WORLD, 0, N_SLOTS, SLOT, epoch, SLOT_OFF, STRIPE, TOTAL, ctas,
               ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))
    assert rc == 0, f"ft_p2p_gather_noalloc returned cudaError {rc}"
    torch.cuda.synchronize(DEV)
    assert native.device_error(reset=True) == 0
    lo, hi = SLOT_OFF + STRIPE, SLOT_OFF + TOTAL  # rank 1's stripe of the slot
    assert torch.equal(a.heap0[lo:hi], src[lo:hi]), "regular entry point did not copy the stripe"
    assert torch.equal(b.heap0, a.heap0), "no-alloc entry point differs from the regular one"
    assert int(b.acks[1][0 * N_SLOTS + SLOT]) == epoch and int(a.acks[1][0 * N_SLOTS + SLOT]) == epoch


def test_noalloc_gather_matches_regular_twice():
    _run_pair(epoch=5, ctas=16)
    _run_pair(epoch=6, ctas=7)  # second call: shared counters must have been cleared/reset


def test_noalloc_gather_rejects_out_of_range():
    f = _fn()
    z = (ctypes.c_uint64 * 1)(0)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    assert f(z, z, z, 1, 0, 257, 0, 1, 0, 256, 256, 1, stream) != 0   # more slots than the array holds
    assert f(z, z, z, 1, 0, 4, 300, 1, 0, 256, 256, 1, stream) != 0   # slot outside range
    assert f(z, z, z, 9, 0, 4, 0, 1, 0, 256, 256, 1, stream) != 0     # too many ranks
