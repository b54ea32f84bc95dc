"""``python -m quantaweave_b200.train``: the training CLI (see ``training.trainer``)."""

from .training.trainer import main

if __name__ == "__main__":
    main()
