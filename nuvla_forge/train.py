"""``python -m nuvla_forge.train``: the training entry point (same flags and presets)."""

import os

from nuvla_forge_b200.train import Trainer, apply_preset, build_args, main  # noqa: F401

if __name__ == "__main__":
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    main()
