import numpy as np
import pytest
import torch

from scirs_b200.utils import memory_efficient as M


def test_mmap_and_chunked_ops(tmp_path):
    data = torch.arange(40, dtype=torch.float32).view(10, 4)
    m = M.create_mmap(str(tmp_path / "a.mmap"), data)
    r = M.open_mmap(str(tmp_path / "a.mmap"), (10, 4), np.float32)
    assert torch.equal(r.to_tensor(2, 5), data[2:5])
    m.write(0, torch.ones(2, 4))
    m.flush()
    assert torch.equal(M.open_mmap(str(tmp_path / "a.mmap"), (10, 4)).to_tensor(0, 2), torch.ones(2, 4))
    with pytest.raises(ValueError):
        M.open_mmap(str(tmp_path / "a.mmap"), (100, 4))
    t = M.create_temp_mmap(data)
    assert M.ChunkedArray(t, 3).num_chunks() == 4
    assert torch.equal(M.chunk_wise_op(t, lambda c: c * 2, 3), data * 2)
    assert torch.equal(M.chunk_wise_binary_op(data, t, lambda a, b: a + b, 4), data * 2)
    s = M.chunk_wise_reduce(t, lambda c: c.sum(0), lambda parts: torch.stack(parts).sum(0), 3)
    assert torch.allclose(s, data.sum(0))
    got = torch.cat(list(M.stream_to_device(t, 4, "cpu")))
    assert torch.equal(got, data)
