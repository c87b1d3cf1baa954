"""``python -m nuvla_forge.bench.report``."""

from nuvla_forge_b200.bench.report import main

if __name__ == "__main__":
    main()
