"""Trainer.Train's loop (pkg/train/trainer.go:508-551) and the dataset
(pkg/train/dataset.go) on the host, with a fake trainer standing in for the
device: log lines every LogInterval steps with the average of the losses
since the last one, SaveCheckpoint every SaveInterval steps and at the end,
windows shifted by one."""
import numpy as np
import pytest

from gollama_b200.train import NewDataLoader, NewDataset, TrainConfig, train_loop


class FakeTrainer:
    def __init__(self, cfg):
        self.Config, self.step, self.saves = cfg, 0, []
        self.totalLoss, self.lossCount = np.float32(0), 0

    def TrainStep(self, inputs, targets):
        assert np.array_equal(inputs[:, 1:], targets[:, :-1])
        self.step += 1
        loss = np.float32(10.0 / self.step)
        self.totalLoss = np.float32(self.totalLoss + loss)
        self.lossCount += 1
        return float(loss)

    def last_stats(self):
        return 0.0, 3e-4, self.step

    def SaveCheckpoint(self):
        self.saves.append(self.step)
        return f"{self.Config.SavePath}/checkpoint_{self.step}.bin"


def test_train_loop_cadence(tmp_path):
    cfg = TrainConfig(MaxSteps=25, LogInterval=10, SaveInterval=20, SavePath=str(tmp_path / "ck"), BatchSize=3,
                      BlockSize=8)
    t = FakeTrainer(cfg)
    loader = NewDataLoader(NewDataset(np.arange(100), 8), 3, True, 5)
    lines = []
    train_loop(t, loader, lines.append)
    assert t.step == 25 and t.saves == [20, 25]
    assert (tmp_path / "ck").is_dir()
    logged = [ln for ln in lines if ln.startswith("step ")]
    assert [int(ln.split()[1]) for ln in logged] == [10, 20]
    want_avg = np.float32(sum(np.float32(10.0 / s) for s in range(11, 21))) / np.float32(10)
    assert f"(avg: {want_avg:.4f})" in logged[1]
    assert lines[-1] == "Training complete! Final step: 25"


def test_empty_batch_raises(tmp_path):
    cfg = TrainConfig(MaxSteps=3, SavePath=str(tmp_path))
    loader = NewDataLoader(NewDataset(np.arange(9), 8), 2, True, 0)  # 9 tokens: no window fits
    with pytest.raises(ValueError):
        train_loop(FakeTrainer(cfg), loader, lambda s: None)


def test_dataset_windows():
    ds = NewDataset(np.arange(50), 16)
    assert ds.Len() == 34
    x, y = ds.GetBatch(64, np.random.default_rng(1))
    assert x.shape == y.shape == (64, 16)
    assert np.array_equal(y, x + 1)
    assert x[:, 0].min() >= 0 and x[:, 0].max() < 50 - 16 - 1
    assert NewDataset(np.arange(16), 16).GetBatch(2, np.random.default_rng(0)) == (None, None)
