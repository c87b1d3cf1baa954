"""``python -m nuvla_forge.bench.bench_dataloader``."""

from nuvla_forge_b200.bench.bench_dataloader import main

if __name__ == "__main__":
    main()
