"""``python -m nuvla_forge.bench.bench_comms``."""

from nuvla_forge_b200.bench.bench_comms import main

if __name__ == "__main__":
    main()
