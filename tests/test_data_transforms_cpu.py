import pytest
import torch

from scirs_b200.data import transforms as T
from scirs_b200.data.loader import InMemoryDataset

D = torch.float64


def test_scalers_onehot_compose():
    x = torch.tensor([[1.0, 10.0], [3.0, 10.0], [5.0, 10.0]], dtype=D)
    s = T.StandardScaler().fit(x)
    z = s.transform(x)
    assert torch.allclose(z[:, 0], torch.tensor([-1.2247, 0.0, 1.2247], dtype=D), atol=1e-4)
    assert torch.allclose(z[:, 1], torch.zeros(3, dtype=D))  # zero std divides by 1
    assert torch.allclose(s.inverse_transform(z), x)
    ps = T.StandardScaler(fit_per_sample=True).fit_transform(x)
    assert torch.allclose(ps.mean(1), torch.zeros(3, dtype=D), atol=1e-12)
    mm = T.MinMaxScaler((-1.0, 1.0)).fit_transform(x)
    assert torch.allclose(mm[:, 0], torch.tensor([-1.0, 0.0, 1.0], dtype=D)) and torch.all(mm[:, 1] == -1.0)
    oh = T.OneHotEncoder(3).transform(torch.tensor([[2], [0]]))
    assert torch.equal(oh, torch.tensor([[0, 0, 1], [1, 0, 0]], dtype=D))
    with pytest.raises(ValueError):
        T.OneHotEncoder(2).transform(torch.tensor([2]))
    c = T.ComposeTransform([T.StandardScaler(), T.MinMaxScaler()]).fit(x)
    assert float(c.transform(x)[:, 0].max()) == 1.0


def test_datasets_and_splits(tmp_path):
    p = tmp_path / "d.csv"
    p.write_text("a,b,label\n1,2,0\n3,4,1\n5,6,0\n")
    ds = T.CSVDataset(str(p))
    assert len(ds) == 3 and torch.equal(ds.get(1)[0], torch.tensor([3.0, 4.0], dtype=D))
    sub = T.SubsetDataset(ds, [2, 0])
    assert len(sub) == 2 and float(sub.get(0)[0][0]) == 5.0
    tr = T.TransformedDataset(ds, feature_transform=lambda f: f * 2)
    assert torch.equal(tr.get(0)[0], torch.tensor([2.0, 4.0], dtype=D))
    x, y = torch.arange(10.0)[:, None], torch.arange(10.0)
    xt, xv, yt, yv = T.train_val_split(x, y, 0.3, shuffle=True, seed=1)
    assert xt.shape[0] == 7 and xv.shape[0] == 3 and sorted(torch.cat([yt, yv]).tolist()) == list(range(10))
    with pytest.raises(ValueError):
        T.train_val_split(x, y, 1.0)
    folds = T.KFold(3).split(10)
    assert [len(te) for _, te in folds] == [4, 3, 3] and sorted(sum((te for _, te in folds), [])) == list(range(10))
    assert all(set(tr_).isdisjoint(te) and len(tr_) + len(te) == 10 for tr_, te in folds)
    assert T.KFold(3, shuffle=True, random_state=5).split(10) == T.KFold(3, shuffle=True, random_state=5).split(10)
    b = T.create_batches(x, y, 4)
    assert [bx.shape[0] for bx, _ in b] == [4, 4, 2]
    assert isinstance(InMemoryDataset(x, y), object)
