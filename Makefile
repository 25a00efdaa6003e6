.PHONY: help build test ci test-gpu smoke bench bench-cpu clean

NPROC ?= 4

help:
	@echo "make build      compile the sm_100a kernels into minidist/_lib/libminidist_cuda.so"
	@echo "make test       CPU correctness suite (Gloo, no GPU needed)"
	@echo "make ci         what CI runs: lint, CPU suite, trainer smoke (tests/run_tests.sh)"
	@echo "make test-gpu   GPU tier (kernel numerics, fused model, multi-GPU)"
	@echo "make smoke      3-D parallel trainer smoke test on Gloo"
	@echo "make bench      headline benchmark (bench.py) on 1 GPU"
	@echo "make bench-cpu  benchmark suite on Gloo/CPU (exercises code, not performance)"

build:
	python -m minidist._build

test:
	python -m pytest tests -q -m "not gpu"

ci:
	tests/run_tests.sh

test-gpu: build
	python -m pytest tests -q -m gpu

smoke:
	python -m torch.distributed.run --nnodes=1 --nproc-per-node=4 --master-addr=127.0.0.1 \
		examples/train_gpt.py --tp 2 --pp 2 --strategy none --microbatches 4 \
		--layers 4 --embd 128 --heads 4 --vocab 1024 --seq-len 64 --batch-size 8 --steps 4 --backend gloo

bench: build
	python bench.py

bench-cpu:
	BACKEND=gloo NPROC=$(NPROC) benchmarks/run_all.sh

clean:
	rm -rf .pytest_cache minidist/_lib/obj
