"""Training launcher: ``python train.py --task train ...`` or under torchrun / run.sh."""
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from centrifuge_b200.train import main  # noqa: E402

if __name__ == "__main__":
    sys.exit(main())
