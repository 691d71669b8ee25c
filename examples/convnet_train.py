"""Train a small ConvNet with the Trainer (the reference's examples/convnet_train.rs, same data):
Conv2d(1->4, 3x3, no padding) -> ReLU -> MaxPool2d(2) -> Flatten -> Linear(16 -> 2) on 8 synthetic 6x6
images whose class is a bright corner. Run: ``python examples/convnet_train.py`` from the repository
root (with the repository on ``PYTHONPATH``)."""
import torch

from brain_b200.nn import Conv2d, Flatten, Linear, MaxPool2d, ReLU, Sequential
from brain_b200.train import Batch, TrainerBuilder


def main():
    imgs = torch.full((8, 1, 6, 6), 0.05)
    for i in range(4):
        imgs[i, 0, 0, 0], imgs[i, 0, 0, 1], imgs[i, 0, 1, 0] = 3.0 + 0.1 * i, 3.0, 3.0
        imgs[4 + i, 0, 5, 5], imgs[4 + i, 0, 5, 4], imgs[4 + i, 0, 4, 5] = 3.0 + 0.1 * i, 3.0, 3.0
    batches = [Batch(imgs, torch.tensor([0, 0, 0, 0, 1, 1, 1, 1]))]
    torch.manual_seed(0)
    model = Sequential(Conv2d(1, 4, 3), ReLU(), MaxPool2d(2, 2), Flatten(), Linear(4 * 2 * 2, 2))
    trainer = TrainerBuilder().model(model).learning_rate(0.1).build()
    before = trainer.evaluate(batches)
    after = trainer.fit(batches, epochs=20)
    print(f"initial loss {before[0]:.4f} accuracy {before[1]:.2f}; after 20 epochs loss {after.loss:.4f}, "
          f"final-epoch accuracy {after.history[-1].accuracy:.2f}")
    return before, after, trainer.evaluate(batches)


if __name__ == "__main__":
    main()
