#!/usr/bin/env python
"""OLMo checkpoint -> ``hf_olmo`` layout: ``config.json``, weights under the ``model.`` key prefix, tokenizer files, so that
``AutoModelForCausalLM.from_pretrained(dir)`` works once ``hf_olmo`` is imported.

    python hf_olmo/convert_olmo_to_hf.py --checkpoint-dir CKPT [--destination-dir OUT] [--tokenizer tok.json]
                                         [--keep-olmo-artifacts] [--ignore-olmo-compatibility] [--pytorch-bin]

``CKPT`` and ``OUT`` may be local folders or URLs of any storage scheme the framework knows (``s3://``, ``r2://``, ``gs://``,
``weka://``): a remote checkpoint is fetched into a temporary folder first, a remote destination is uploaded to at the end.
Sharded checkpoints (this framework's or the reference's layouts) are unsharded on the host first.  The steps are
functions of their own so that they can be driven from other tools; they carry the names of the reference's converter
(``hf_olmo/convert_olmo_to_hf.py:34-316``).
"""
import argparse
import logging
import os
import shutil
import sys
import tempfile
from pathlib import Path
from typing import Iterable, List, Optional

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))

logger = logging.getLogger(__name__)

#: what only this framework (not ``transformers``) reads in a checkpoint folder
OLMO_ARTIFACTS = ("config.yaml", "model.pt", "model.olmo.safetensors", "optim.pt", "train.pt", "optim", "model", "train", "metadata.yaml")


def longest_common_prefix(strs: Iterable[str]) -> str:
    """The longest string every element starts with (empty for an empty input)."""
    items: List[str] = sorted(strs)
    if not items:
        return ""
    first, last = items[0], items[-1]  # after sorting, these two differ the most
    n = 0
    while n < min(len(first), len(last)) and first[n] == last[n]:
        n += 1
    return first[:n]


def download_s3_directory(url: str, local_dir: str, ignore: Optional[str] = None) -> int:
    """Copy every file below a remote prefix (any registered scheme, not just S3) into ``local_dir``, keeping relative
    paths; names containing ``ignore`` are skipped.  Returns the number of files copied."""
    from olmo_b200.util import file_size, get_bytes_range, list_files

    files = list_files(url)
    root = longest_common_prefix(files) if len(files) > 1 else url.rstrip("/") + "/"
    root = root[: root.rfind("/") + 1]
    copied = 0
    for remote in files:
        rel = remote[len(root):]
        if ignore and ignore in rel:
            continue
        target = Path(local_dir) / rel
        target.parent.mkdir(parents=True, exist_ok=True)
        size, chunk = file_size(remote), 64 << 20
        with open(target, "wb") as f:
            for off in range(0, size, chunk):
                f.write(get_bytes_range(remote, off, min(chunk, size - off)))
        copied += 1
    return copied


def make_local_checkpoint(checkpoint_dir: str) -> str:
    """A local folder holding the checkpoint: the folder itself, or a temporary copy of a remote one (optimizer and
    trainer state are not fetched; the conversion does not read them)."""
    from olmo_b200.util import is_url

    if not is_url(checkpoint_dir):
        return checkpoint_dir
    local = tempfile.mkdtemp(prefix="olmo_ckpt_")
    n = download_s3_directory(checkpoint_dir, local, ignore="optim")
    if n == 0:
        raise FileNotFoundError(f"nothing found under {checkpoint_dir}")
    logger.info("fetched %d files of %s into %s", n, checkpoint_dir, local)
    return local


def maybe_unshard(checkpoint_dir: str) -> None:
    """Make sure ``checkpoint_dir`` holds unsharded weights (``model.pt`` / ``model.safetensors``), gathering a sharded
    checkpoint of any known layout on the host when it does not."""
    src = Path(checkpoint_dir)
    if (src / "model.pt").is_file() or (src / "model.safetensors").is_file():
        return
    from olmo_b200.checkpoint import build_sharded_checkpointer
    from olmo_b200.config import TrainConfig

    import torch

    cfg = TrainConfig.load(src / "config.yaml", validate_paths=False)
    model_state, _, _ = build_sharded_checkpointer(cfg).unshard_checkpoint(src, load_optimizer_state=False, load_trainer_state=False)
    torch.save(model_state, src / "model.pt")


def write_config(checkpoint_dir: str) -> None:
    """``config.json`` from the model section of ``config.yaml``."""
    from olmo_b200.config import TrainConfig
    from olmo_b200.hf.configuration import OLMoConfig

    model = TrainConfig.load(Path(checkpoint_dir) / "config.yaml", validate_paths=False).model
    OLMoConfig(**model.asdict()).save_pretrained(checkpoint_dir)


def write_model(checkpoint_dir: str, ignore_olmo_compatibility: bool = False, safe_serialization: bool = False) -> None:
    """The weights under the ``model.`` prefix, as ``pytorch_model.bin`` (or ``model.safetensors``); with
    ``ignore_olmo_compatibility`` the framework's own weight file is removed afterwards."""
    import torch

    from olmo_b200.hf.convert import _strip_prefixes, load_unsharded_model_state

    src = Path(checkpoint_dir)
    state = {f"model.{k}": v.contiguous() for k, v in _strip_prefixes(load_unsharded_model_state(src)).items()}
    if safe_serialization:
        from safetensors.torch import save_file

        if (src / "model.safetensors").is_file():  # the framework's own flavour of the same name
            (src / "model.safetensors").rename(src / "model.olmo.safetensors")
        save_file(state, str(src / "model.safetensors"), metadata={"format": "pt"})
    else:
        torch.save(state, src / "pytorch_model.bin")
    if ignore_olmo_compatibility:
        (src / "model.pt").unlink(missing_ok=True)
        (src / "model.olmo.safetensors").unlink(missing_ok=True)


def write_tokenizer(checkpoint_dir: str, tokenizer_path: Optional[str] = None) -> None:
    """Tokenizer files for ``AutoTokenizer`` (vocabulary named in ``config.yaml`` unless ``tokenizer_path`` is given)."""
    from olmo_b200.config import TrainConfig
    from olmo_b200.hf.convert import _copy_tokenizer

    cfg = TrainConfig.load(Path(checkpoint_dir) / "config.yaml", validate_paths=False)
    _copy_tokenizer(cfg, Path(checkpoint_dir), tokenizer_path)


def fix_tokenizer(checkpoint_dir: str, tokenizer_name_or_path: Optional[str] = None) -> None:
    """Point ``config.yaml`` at a tokenizer that can be found: the override when given, otherwise the configured file when
    it exists, otherwise the packaged tokenizer of the same file name."""
    from olmo_b200.config import TrainConfig

    path = Path(checkpoint_dir) / "config.yaml"
    cfg = TrainConfig.load(path, validate_paths=False)
    ident = tokenizer_name_or_path or cfg.tokenizer.identifier
    if tokenizer_name_or_path is None and not Path(ident).is_file():
        packaged = f"tokenizers/{Path(ident).name}"
        try:
            from olmo_data.data import is_data_file

            if is_data_file(packaged):
                ident = packaged
        except ImportError:
            pass
    if ident != cfg.tokenizer.identifier:
        cfg.tokenizer.identifier = ident
        cfg.save(path)


def convert_checkpoint(checkpoint_dir: str, ignore_olmo_compatibility: bool = False, safe_serialization: bool = False) -> None:
    """All three outputs in place."""
    write_config(checkpoint_dir)
    write_model(checkpoint_dir, ignore_olmo_compatibility=ignore_olmo_compatibility, safe_serialization=safe_serialization)
    write_tokenizer(checkpoint_dir)


def upload_local_checkpoint(local_checkpoint_dir: str, destination_dir: str) -> None:
    """Put the converted folder where it was asked for: nothing to do when it already is there, a copy for another local
    folder, an upload for a URL."""
    from olmo_b200.util import is_url, upload

    if os.path.abspath(local_checkpoint_dir) == os.path.abspath(destination_dir) and not is_url(destination_dir):
        return
    for path in sorted(Path(local_checkpoint_dir).rglob("*")):
        if not path.is_file():
            continue
        rel = path.relative_to(local_checkpoint_dir)
        if is_url(destination_dir):
            upload(path, f"{destination_dir.rstrip('/')}/{rel}", save_overwrite=True)
        else:
            target = Path(destination_dir) / rel
            target.parent.mkdir(parents=True, exist_ok=True)
            shutil.copyfile(path, target)


def main(argv: Optional[List[str]] = None) -> str:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--checkpoint-dir", required=True, help="folder or URL of the OLMo checkpoint")
    ap.add_argument("--destination-dir", default=None, help="folder or URL for the result (default: the checkpoint folder itself)")
    ap.add_argument("--tokenizer", default=None, help="tokenizer.json to ship instead of the one named in config.yaml")
    ap.add_argument("--keep-olmo-artifacts", action="store_true", help="leave config.yaml, model.pt and the state folders in the result")
    ap.add_argument("--ignore-olmo-compatibility", action="store_true", help="drop the framework's own weight file while converting")
    ap.add_argument("--pytorch-bin", action="store_true", help="accepted for compatibility (pytorch_model.bin is the default)")
    ap.add_argument("--safetensors", action="store_true", help="write model.safetensors instead of pytorch_model.bin")
    ap.add_argument("--logger-level", default="warning")
    args = ap.parse_args(argv)
    logging.basicConfig()
    logger.setLevel(logging.getLevelName(args.logger_level.upper()))

    destination = args.destination_dir or args.checkpoint_dir
    local = make_local_checkpoint(args.checkpoint_dir)
    work = local
    same_place = os.path.abspath(local) == os.path.abspath(destination)
    if not same_place and local == args.checkpoint_dir:
        # converting into another folder: work on a copy so that the source checkpoint stays as it is
        work = tempfile.mkdtemp(prefix="olmo_hf_")
        for name in os.listdir(local):
            if "optim" in name or name == "train" or name == "train.pt":
                continue
            src = os.path.join(local, name)
            (shutil.copytree if os.path.isdir(src) else shutil.copyfile)(src, os.path.join(work, name))
    maybe_unshard(work)
    fix_tokenizer(work, args.tokenizer)
    convert_checkpoint(work, args.ignore_olmo_compatibility, safe_serialization=args.safetensors)
    if not args.keep_olmo_artifacts:
        for name in OLMO_ARTIFACTS:
            path = Path(work) / name
            if path.is_dir():
                shutil.rmtree(path, ignore_errors=True)
            else:
                path.unlink(missing_ok=True)
    upload_local_checkpoint(work, destination)
    print(f"Converted checkpoint saved to {destination}")
    return destination


if __name__ == "__main__":
    main()
