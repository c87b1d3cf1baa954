.PHONY: build test test-gpu bench bench-all bench-comms train-ab report probe clean
NGPU ?= 2

build:
	python -m nuvla_forge_b200._build

test:
	python -m pytest tests -m "not gpu" -q

test-gpu: build
	python -m pytest tests -m gpu -q

bench: build
	python bench.py
	python -m nuvla_forge_b200.bench.bench_kernels
	python -m nuvla_forge_b200.bench.bench_dataloader

bench-all: build
	python -m nuvla_forge_b200.bench.run_all

bench-comms: build
	python -m torch.distributed.run --nproc-per-node $(NGPU) --master-addr 127.0.0.1 -m nuvla_forge_b200.bench.bench_comms

train-ab: build
	python -m torch.distributed.run --nproc-per-node $(NGPU) --master-addr 127.0.0.1 -m nuvla_forge_b200.train --preset baseline --steps 50
	python -m torch.distributed.run --nproc-per-node $(NGPU) --master-addr 127.0.0.1 -m nuvla_forge_b200.train --preset optimised --steps 50

report:
	python -m nuvla_forge_b200.bench.report

probe:
	python -m nuvla_forge_b200.utils.probe

clean:
	rm -rf nuvla_forge_b200/_lib/obj RESULTS.md .pytest_cache
