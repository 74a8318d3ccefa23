"""Worker for tests/test_failure_cpu.py's elastic-restart test, run under
``torch.distributed.run --max-restarts 1``: the training entry point with a
host-side fault. In the first attempt (TORCHELASTIC_RESTART_COUNT 0) rank 1
raises before its third step; the agent restarts every rank, which resume
from the last checkpoint. No device is involved.

    python -m torch.distributed.run --nproc-per-node 2 --max-restarts 1 tests/elastic_worker.py <train args>
"""
import os
import sys

from dion_b200 import train
from dion_b200.integration.trainer import Trainer


def _inject() -> None:
    if int(os.environ.get("TORCHELASTIC_RESTART_COUNT", "0")) != 0 or os.environ.get("RANK") != "1":
        return
    step = Trainer.train_step

    def failing(self, tokens, labels):
        if self.step_idx == 2:
            raise RuntimeError("injected host-side failure before step 3")
        return step(self, tokens, labels)

    Trainer.train_step = failing


if __name__ == "__main__":
    _inject()
    train.main(sys.argv[1:])
