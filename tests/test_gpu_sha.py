"""SHA-256 on the GPU: bit-exact against OpenSSL's digests and the
reference's compute_block_id (golden), at every padding boundary, for
aligned and misaligned blocks, alone and in ragged batches."""
import hashlib

import numpy as np
import pytest
import torch

import oracle
from cascade_b200 import _lib
from cascade_b200 import cascade_cpp as cc
from cascade_b200 import workloads
from gpu_util import DEV, addr_table, size_table, stream, to_dev
from make_golden import SHA_LENGTHS, STORED_MAX, sha_input

pytestmark = pytest.mark.gpu


def _inputs(d):
    out = []
    for i, n in enumerate(SHA_LENGTHS):
        if n <= STORED_MAX:
            off = int(d["offsets"][i])
            out.append(d["data"][off:off + n])
        else:
            out.append(sha_input(n))
    return out


def _gpu_digests(tensors):
    ptrs = addr_table(tensors)
    sizes = size_table([t.numel() for t in tensors])
    dig = torch.empty(32 * len(tensors), dtype=torch.uint8, device=DEV)
    _lib.call("cascade_sha256_batch", ptrs.data_ptr(), sizes.data_ptr(),
              len(tensors), dig.data_ptr(), stream())
    torch.cuda.synchronize()
    return dig.view(-1, 32).cpu().numpy()


@pytest.mark.parametrize("misalign", [0, 1, 2, 3, 5, 8, 13])
def test_sha_golden_ragged_batch(sha_cases, misalign):
    xs = _inputs(sha_cases)
    ts = [to_dev(x, pad_front=(misalign * (i + 1)) % 16) for i, x in enumerate(xs)]
    d = _gpu_digests(ts)
    for i, x in enumerate(xs):
        assert d[i].tobytes() == sha_cases["digests"][i].tobytes(), len(x)
        assert d[i][:16].tobytes().hex() == str(sha_cases["block_ids"][i])


def test_sha_empty_batch_is_noop():
    _lib.call("cascade_sha256_batch", 0, 0, 0, 0, stream())


def test_compute_block_id_host_buffer(sha_cases):
    xs = _inputs(sha_cases)
    for i in (0, 1, 55, 56, 63, 64, 65, 119, 120, 300, len(xs) - 1):
        assert cc.compute_block_id(xs[i]) == str(sha_cases["block_ids"][i])
    assert cc.compute_block_id(b"abc") == hashlib.sha256(b"abc").hexdigest()[:32]


def test_compute_block_ids_kv_blocks():
    blocks = workloads.kv_blocks_np(8, 11, layers=32)   # 8 x 2 MiB
    dev = torch.from_numpy(blocks).to(DEV)
    ids = cc.compute_block_ids([dev[i] for i in range(8)])
    assert ids == [oracle.block_id(b) for b in blocks]
    full = cc.sha256_batch([dev[i] for i in range(8)]).cpu().numpy()
    for i in range(8):
        assert full[i].tobytes() == hashlib.sha256(blocks[i].tobytes()).digest()


@pytest.mark.parametrize("n", [4096, 8192, 12288])
def test_sha_many_chains_sample_checked(n):
    # One warp pair per SM (4096), two per SM (8192) and the shared-scheduler
    # form (12288): ragged sizes, every 7th block unaligned; spot-checked
    # against OpenSSL across the batch, the last blocks included.
    s = 4096
    g = torch.Generator(device=DEV)
    g.manual_seed(5)
    data = torch.randint(0, 256, (n, s + 16), dtype=torch.uint8, device=DEV,
                         generator=g)
    sizes = [s - (i % 193) for i in range(n)]
    offs = [(i % 13) if i % 7 == 0 else 0 for i in range(n)]
    blocks = [data[i, offs[i]:offs[i] + sizes[i]] for i in range(n)]
    d = _gpu_digests(blocks)
    host = data.cpu().numpy()
    check = sorted(set(list(range(0, n, n // 40)) + [1, 7, 31, 32, 33, n - 2, n - 1]))
    for i in check:
        want = hashlib.sha256(host[i, offs[i]:offs[i] + sizes[i]].tobytes()).digest()
        assert d[i].tobytes() == want, i
    if n != 4096:
        return
    # size-independent property: equal blocks, equal digests
    d2 = _gpu_digests([blocks[7], blocks[7], blocks[8]])
    assert (d2[0] == d2[1]).all() and not (d2[0] == d2[2]).all()
    assert (d2[0] == d[7]).all()
