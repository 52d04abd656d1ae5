"""Package data of the framework: tokenizer files, evaluation datasets and request dumps live below this folder (or below
``OLMO_DATA_DIR``, which wins).  See ``olmo_data/README.md`` for the layout."""
