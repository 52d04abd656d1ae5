# Convenience targets; everything they do is a plain python / pytest command.
.PHONY: build test test-gpu bench configs check-cpu-install check-cuda-install

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
