# Makefile - build and convenience targets.  The native extension (every
# sm_100a kernel and the C++ ring runtime) is built in place by setup.py.
CONFIG ?= benchmark.env
-include $(CONFIG)
PYTHON ?= python3

.PHONY: all build comm attention check-attention-correctness test test-gpu print-config clean help

all: build

build:
	$(PYTHON) setup.py build_ext --inplace

# The comm and attention programs in bin/ share the one extension.
comm attention: build

check-attention-correctness: build
	BUILD=0 ./check_attention_correctness.sh

test:
	$(PYTHON) -m pytest tests -q -m "not gpu"

test-gpu: build
	$(PYTHON) -m pytest tests -q -m gpu

print-config:
	@echo "CONFIG=$(CONFIG)"
	@echo "LAUNCHER=$(LAUNCHER)"
	@echo "NP_LIST=$(NP_LIST)"
	@echo "BACKENDS=$(BACKENDS)"
	@echo "ATTENTION_BACKENDS=$(ATTENTION_BACKENDS)"
	@echo "COMM_SIZES=$(COMM_SIZES)"
	@echo "ATTENTION_SIZES=$(ATTENTION_SIZES)"
	@echo "NVCC=$$(command -v nvcc)"

clean:
	rm -rf build ring_attention_benchmark_b200/_C*.so

help:
	@echo "targets: build (default) comm attention check-attention-correctness test test-gpu print-config clean"
