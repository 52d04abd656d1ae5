# Convenience targets; everything they do is a plain python / pytest command.
.PHONY: build test test-gpu bench configs check-cpu-install check-cuda-install run-checks image test-image show-image

IMAGE ?= olmo-b200

build:
	python -c "import __graft_entry__ as g; g.build()"

test:
	python -m pytest tests/ -q -m "not gpu"

test-gpu:
	python -m pytest tests/ -q -m gpu

bench:
	python bench.py

configs:
	python -m olmo_b200.recipes --write configs

check-cpu-install:
	python -c "from olmo_b200 import check_install; check_install(cuda=False)"

check-cuda-install:
	python -c "from olmo_b200 import check_install; check_install(cuda=True)"

# Style and type checks run only when their tool is installed; the CPU test suite always runs.
run-checks:
	@for tool in "isort --check ." "black --check ." "ruff check ." "mypy olmo_b200"; do \
		if command -v $${tool%% *} >/dev/null 2>&1; then echo "+ $$tool"; $$tool || exit 1; else echo "(skipped: $${tool%% *} is not installed)"; fi; \
	done
	CUDA_VISIBLE_DEVICES='' python -m pytest -q -m "not gpu" tests/

# The one image serves training, serving and the test suite (its default command runs the CPU tests).
image:
	docker build -f docker/Dockerfile -t $(IMAGE) .

test-image: image
	docker run --rm $(IMAGE)

show-image:
	@echo $(IMAGE)
