"""``python -m nuvla_forge.bench.bench_kernels``."""

from nuvla_forge_b200.bench.bench_kernels import main

if __name__ == "__main__":
    main()
