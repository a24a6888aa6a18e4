"""micro_engram.train: `torchrun -m micro_engram.train cfg.yaml`."""
