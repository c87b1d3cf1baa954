"""``nuvla_forge.bench``: the benchmark entry points."""
