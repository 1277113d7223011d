# Build and check targets (the reference's CI, .github/workflows/ci.yml:31-56,
# and scripts/verify.sh, restated for this framework).
#
#   make build      host library and sm_100a kernels, in-tree
#   make build-host host library only (machines without nvcc)
#   make test       CPU test suite (no GPU needed)
#   make test-gpu   GPU test suite (needs a B200)
#   make sanitize   host library under ASan + UBSan and TSan; bounds-checked
#                   kernel build compiles
#   make verify     regenerate the verification artifacts and check each
#                   against the reference's committed result (verification/)
#   make check      build, compile-check, test, sanitize, verify (what CI runs)
PYTHON ?= python
VERIFY_DIR ?= verification

.PHONY: build build-host compile test test-gpu sanitize verify check clean

build:
	$(PYTHON) setup.py build_ext --inplace

build-host:
	NGL_SKIP_CUDA=1 $(PYTHON) setup.py build_ext --inplace

compile:
	$(PYTHON) -m compileall -q mini_nangila_b200 nangila_ddp tests bench.py __graft_entry__.py

test:
	$(PYTHON) -m pytest tests -x -q -m "not gpu"

test-gpu:
	$(PYTHON) -m pytest tests -x -q -m gpu

sanitize:
	$(PYTHON) -m pytest tests/test_sanitizers.py tests/test_debug_build.py -x -q

verify:
	$(PYTHON) -m mini_nangila_b200.apps.verify --out $(VERIFY_DIR) --skip-tests

check: build compile test sanitize verify

clean:
	rm -rf build _build mini_nangila_b200/*.so
