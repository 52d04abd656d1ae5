"""
Host-side utilities: logging, CLI helpers, storage back ends, small iterator tools.

Covers the capabilities of the reference's ``olmo/util.py:52-943`` with a different structure:
storage is a registry of :class:`StorageBackend` objects keyed by URL scheme (local files and
``file://`` always; ``http(s)://`` through ``requests``; ``s3://``, ``r2://``, ``weka://`` through
``boto3`` and ``gs://`` through ``google-cloud-storage`` when those packages are importable).
The module-level functions :func:`file_size`, :func:`get_bytes_range`, :func:`upload` and
:func:`find_latest_checkpoint` dispatch on the scheme.
"""
from __future__ import annotations

import gzip
import io
import json
import logging
import os
import re
import socket
import sys
import time
import warnings
from datetime import datetime
from enum import Enum
from pathlib import Path
from queue import Queue
from threading import Thread
from typing import Any, Callable, Dict, Iterable, Iterator, List, MutableMapping, Optional, Sequence, Tuple, Union
from urllib.parse import urlparse

from .aliases import PathOrStr
from .exceptions import (
    OLMoCliError,
    OLMoEnvironmentError,
    OLMoError,
    OLMoNetworkError,
    OLMoThreadError,
)

__all__ = [
    "StrEnum",
    "LogFilterType",
    "log_extra_field",
    "setup_logging",
    "install_excepthook",
    "RichHandler",
    "excepthook",
    "get_progress_bar",
    "save_hf_dataset_to_disk",
    "filter_warnings",
    "set_env_variables",
    "prepare_cli_environment",
    "clean_opt",
    "positional_args",
    "wait_for",
    "is_url",
    "dir_is_empty",
    "resource_path",
    "file_size",
    "upload",
    "get_bytes_range",
    "find_latest_checkpoint",
    "list_files",
    "delete_file",
    "StorageBackend",
    "register_storage_backend",
    "default_thread_count",
    "pass_through_fn",
    "threaded_generator",
    "roundrobin",
    "add_cached_path_clients",
    "flatten_dict",
    "load_hf_dataset",
    "load_oe_eval_requests",
]

log = logging.getLogger(__name__)


class StrEnum(str, Enum):
    """String-valued enum whose ``str()`` is its value (so it formats cleanly in paths and logs)."""

    def __str__(self) -> str:
        return self.value

    def __repr__(self) -> str:
        return f"'{str(self)}'"


class LogFilterType(StrEnum):
    rank0_only = "rank0_only"
    local_rank0_only = "local_rank0_only"
    all_ranks = "all_ranks"


# ---------------------------------------------------------------------------------------------
# Logging (reference: olmo/util.py:69-155, 222-286)
# ---------------------------------------------------------------------------------------------

_log_extra_fields: Dict[str, Any] = {}


def log_extra_field(field_name: str, field_value: Any) -> None:
    """Attach a constant attribute (e.g. ``hostname``) to every log record, or remove it with None."""
    if field_value is None:
        _log_extra_fields.pop(field_name, None)
    else:
        _log_extra_fields[field_name] = field_value


def _rank_env(name: str, default: int = 0) -> int:
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class _RankFilter(logging.Filter):
    """Lets INFO-and-below records through only on the selected ranks; warnings always pass."""

    def __init__(self, kind: LogFilterType):
        super().__init__()
        self.kind = kind

    def filter(self, record: logging.LogRecord) -> bool:
        if record.levelno > logging.INFO or self.kind == LogFilterType.all_ranks:
            return True
        if self.kind == LogFilterType.rank0_only:
            return getattr(record, "global_rank", 0) == 0
        return getattr(record, "local_rank", 0) == 0


def setup_logging(log_filter_type: LogFilterType = LogFilterType.rank0_only) -> None:
    """Configure root logging with rank information injected into every record."""
    log_extra_field("hostname", socket.gethostname())
    log_extra_field("local_rank", _rank_env("LOCAL_RANK"))
    log_extra_field("global_rank", _rank_env("RANK"))
    log_extra_field("node_rank", _rank_env("NODE_RANK"))

    base_factory = logging.getLogRecordFactory()
    if not getattr(base_factory, "_olmo_b200_wrapped", False):

        def factory(*args, **kwargs) -> logging.LogRecord:
            record = base_factory(*args, **kwargs)
            for k, v in _log_extra_fields.items():
                setattr(record, k, v)
            return record

        factory._olmo_b200_wrapped = True  # type: ignore[attr-defined]
        logging.setLogRecordFactory(factory)

    interactive = sys.stdout.isatty() and os.environ.get("OLMo_NONINTERACTIVE", "") == ""
    handler: logging.Handler
    if interactive:
        try:
            handler = _rich_handler()
        except Exception:  # rich missing or console creation failed
            handler = logging.StreamHandler(sys.stdout)
            interactive = False
    else:
        handler = logging.StreamHandler(sys.stdout)
    if not interactive:
        handler.setFormatter(
            logging.Formatter(
                "%(asctime)s\t%(hostname)s:%(local_rank)s\t%(name)s:%(lineno)s\t%(levelname)s\t%(message)s",
                datefmt="%Y-%m-%d %H:%M:%S",
            )
        )
    handler.addFilter(_RankFilter(log_filter_type))
    logging.basicConfig(handlers=[handler], level=logging.INFO, force=True)
    logging.captureWarnings(True)
    logging.getLogger("urllib3").setLevel(logging.ERROR)


class RichHandler(logging.Handler):
    """Log records on a ``rich`` console: time, level, ``[logger:line, rank=…]``, message, and a formatted traceback when
    the record carries one (the look of the reference's handler of this name, ``olmo/util.py:222-286``).  ``rich`` is imported
    when the first record arrives, so the class can be named on machines without it."""

    def __init__(self, level: int = logging.NOTSET, markup: bool = False):
        super().__init__(level=level)
        self.markup = markup

    def emit(self, record: logging.LogRecord) -> None:
        try:
            import rich
            from rich.text import Text

            console = rich.get_console()
            stamp = datetime.fromtimestamp(record.created).strftime("[%Y-%m-%d %X]")
            where = f"{record.name}:{record.lineno}" if record.name != "root" else "root"
            message = record.getMessage()
            console.print(
                Text(stamp, style="log.time", end=" "),
                Text(record.levelname.ljust(8), style="log.level", end=" "),
                Text(f"[{where}, rank={getattr(record, 'local_rank', 0)}]", style="log.path"),
                Text.from_markup(message) if self.markup else Text(message),
            )
            if record.exc_info:
                from rich.traceback import Traceback

                console.print(Traceback.from_exception(*record.exc_info))  # type: ignore[arg-type]
        except Exception:
            self.handleError(record)


def _rich_handler() -> logging.Handler:
    import rich

    rich.reconfigure(width=max(rich.get_console().width, 180), soft_wrap=True)
    return RichHandler()


def excepthook(exctype, value, traceback) -> None:
    """``sys.excepthook`` replacement: command-line mistakes print one line, everything else is logged with its traceback
    (so that it reaches the log handlers of every rank), Ctrl-C keeps Python's own behaviour."""
    if issubclass(exctype, KeyboardInterrupt):
        sys.__excepthook__(exctype, value, traceback)
    elif issubclass(exctype, OLMoCliError):
        print(f"error: {value}", file=sys.stderr)
    elif issubclass(exctype, OLMoError):
        log.critical("%s: %s", exctype.__name__, value, exc_info=(exctype, value, traceback))
    else:
        log.critical("Uncaught %s: %s", exctype.__name__, value, exc_info=(exctype, value, traceback))


_excepthook = excepthook  # earlier name


def install_excepthook() -> None:
    sys.excepthook = excepthook


def get_progress_bar():
    """A ``rich`` progress display for transfers (description, bar, bytes done, rate, time left), as used while
    checkpoint files are fetched (``resource_path(..., progress=...)``)."""
    from rich.progress import BarColumn, DownloadColumn, Progress, TextColumn, TimeRemainingColumn, TransferSpeedColumn

    return Progress(TextColumn("[progress.description]{task.description}"), BarColumn(), DownloadColumn(), TransferSpeedColumn(),
                    TimeRemainingColumn(), transient=True)


def filter_warnings() -> None:
    for msg in (
        "torch.distributed.*_base is a private function and will be deprecated.*",
        "TypedStorage is deprecated.*",
        "Please use DTensor instead.*",
        "failed to load.*",
    ):
        warnings.filterwarnings("ignore", category=UserWarning, message=msg)
    warnings.filterwarnings("ignore", category=FutureWarning, module="torch")


def set_env_variables() -> None:
    os.environ.setdefault("TOKENIZERS_PARALLELISM", "false")


def prepare_cli_environment(log_filter_type: Optional[LogFilterType] = None) -> None:
    """One call that every entry point makes: logging, excepthook, warning filters, env."""
    if log_filter_type is None:
        log_filter_type = LogFilterType(os.environ.get("LOG_FILTER_TYPE", "rank0_only"))
    setup_logging(log_filter_type)
    install_excepthook()
    filter_warnings()
    set_env_variables()


def clean_opt(arg: str) -> str:
    """``--some-flag`` -> ``some_flag=True``; ``--a.b-c=1`` -> ``a.b_c=1`` (value left untouched)."""
    key, sep, val = arg.partition("=")
    if not sep:
        val = "True"
    key = key.strip("-").replace("-", "_")
    return f"{key}={val}"


def positional_args(doc: Optional[str], minimum: int, argv: Optional[Sequence[str]] = None) -> List[str]:
    """The arguments of a small positional-argument script: ``-h`` / ``--help`` prints ``doc`` and exits 0, fewer than
    ``minimum`` arguments print it to stderr and exit 2; otherwise ``argv[1:]`` is returned."""
    args = list(sys.argv[1:] if argv is None else argv)
    if any(a in ("-h", "--help") for a in args):
        print((doc or "").strip())
        raise SystemExit(0)
    if len(args) < minimum:
        print((doc or "").strip(), file=sys.stderr)
        raise SystemExit(2)
    return args


def wait_for(condition: Callable[[], bool], description: str, timeout: float = 10.0) -> None:
    """Poll ``condition`` every half second; raise :class:`TimeoutError` after ``timeout`` seconds."""
    deadline = time.monotonic() + timeout
    while not condition():
        if time.monotonic() > deadline:
            raise TimeoutError(f"{description} timed out")
        time.sleep(0.5)


def is_url(path: PathOrStr) -> bool:
    return re.match(r"[a-z0-9]+://.*", str(path)) is not None


def dir_is_empty(dir: PathOrStr) -> bool:
    d = Path(dir)
    if not d.is_dir():
        return True
    return next(iter(d.iterdir()), None) is None


# ---------------------------------------------------------------------------------------------
# Storage back ends
# ---------------------------------------------------------------------------------------------

_STEP_DIR = re.compile(r"^step(\d+)(-unsharded)?$")


def _pick_latest(names: Iterable[str]) -> Optional[str]:
    """Among ``stepN`` / ``stepN-unsharded`` names choose the highest N; sharded wins a tie."""
    best: Optional[Tuple[int, int, str]] = None
    for name in names:
        m = _STEP_DIR.match(name)
        if m is None:
            continue
        key = (int(m.group(1)), 0 if m.group(2) else 1, name)
        if best is None or key[:2] > best[:2]:
            best = key
    return None if best is None else best[2]


class StorageBackend:
    """Interface for one URL scheme."""

    def file_size(self, url: str) -> int:
        raise NotImplementedError

    def get_bytes_range(self, url: str, start: int, num: int) -> bytes:
        raise NotImplementedError

    def upload(self, source: Path, url: str, save_overwrite: bool = False) -> None:
        raise NotImplementedError(f"upload is not supported for {url}")

    def find_latest_checkpoint(self, url: str) -> Optional[str]:
        raise NotImplementedError(f"find_latest_checkpoint is not supported for {url}")

    def list_files(self, url: str) -> List[str]:
        """Full URLs of every file below the folder / prefix ``url``."""
        raise NotImplementedError(f"listing is not supported for {url}")

    def delete(self, url: str) -> None:
        """Remove one file."""
        raise NotImplementedError(f"delete is not supported for {url}")


class _LocalBackend(StorageBackend):
    @staticmethod
    def _p(url: str) -> str:
        return url[len("file://") :] if url.startswith("file://") else url

    def file_size(self, url: str) -> int:
        return os.stat(self._p(url)).st_size

    def get_bytes_range(self, url: str, start: int, num: int) -> bytes:
        with open(self._p(url), "rb") as f:
            f.seek(start)
            return f.read(num)

    def upload(self, source: Path, url: str, save_overwrite: bool = False) -> None:
        import shutil

        target = Path(self._p(url))
        if target.exists() and not save_overwrite:
            raise FileExistsError(f"{target} already exists; use save_overwrite to replace it")
        target.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(source, target)

    def find_latest_checkpoint(self, url: str) -> Optional[str]:
        root = Path(self._p(url))
        if not root.is_dir():
            return None
        name = _pick_latest(p.name for p in root.iterdir() if p.is_dir())
        return None if name is None else str(root / name)

    def list_files(self, url: str) -> List[str]:
        root = Path(self._p(url))
        return sorted(str(p) for p in root.rglob("*") if p.is_file()) if root.is_dir() else []

    def delete(self, url: str) -> None:
        Path(self._p(url)).unlink(missing_ok=True)


def _retry(fn: Callable[[], Any], what: str, max_attempts: int = 3) -> Any:
    """Run ``fn`` with exponential back-off; FileNotFoundError is never retried."""
    err: Optional[Exception] = None
    for attempt in range(1, max_attempts + 1):
        try:
            return fn()
        except FileNotFoundError:
            raise
        except Exception as e:  # network-level failures of whichever client library
            err = e
            if attempt < max_attempts:
                log.warning("%s failed attempt %d: %s", what, attempt, e)
                time.sleep(min(0.5 * 2**attempt, 3.0))
    raise OLMoNetworkError(f"{what} failed after {max_attempts} attempts") from err


class _HttpBackend(StorageBackend):
    def file_size(self, url: str) -> int:
        import requests

        def go() -> int:
            r = requests.head(url, allow_redirects=True, timeout=30)
            if r.status_code == 404:
                raise FileNotFoundError(url)
            r.raise_for_status()
            size = r.headers.get("content-length")
            if size is None:
                raise OLMoNetworkError(f"no content-length for {url}")
            return int(size)

        return _retry(go, f"HEAD {url}")

    def get_bytes_range(self, url: str, start: int, num: int) -> bytes:
        import requests

        def go() -> bytes:
            r = requests.get(url, headers={"Range": f"bytes={start}-{start + num - 1}"}, timeout=60)
            if r.status_code == 404:
                raise FileNotFoundError(url)
            r.raise_for_status()
            if len(r.content) != num:
                raise OLMoNetworkError(f"expected {num} bytes from {url}, got {len(r.content)}")
            return r.content

        return _retry(go, f"GET {url}", max_attempts=5)


class _S3Backend(StorageBackend):
    """``s3://``, ``r2://`` and ``weka://`` share the S3 protocol; endpoints come from the environment."""

    def __init__(self) -> None:
        self._clients: Dict[str, Any] = {}

    def _client(self, scheme: str):
        if scheme in self._clients:
            return self._clients[scheme]
        try:
            import boto3
            from botocore.config import Config
        except ImportError as e:
            raise OLMoEnvironmentError(f"'{scheme}://' paths need the boto3 package") from e
        kwargs: Dict[str, Any] = {}
        profile = None
        if scheme == "s3":
            profile = os.environ.get("S3_PROFILE")
        elif scheme == "r2":
            profile = os.environ.get("R2_PROFILE")
            endpoint = os.environ.get("R2_ENDPOINT_URL")
            if endpoint is None:
                raise OLMoEnvironmentError("R2 endpoint url is not set; did you forget R2_ENDPOINT_URL?")
            kwargs["endpoint_url"] = endpoint
        elif scheme == "weka":
            profile = os.environ.get("WEKA_PROFILE")
            endpoint = os.environ.get("WEKA_ENDPOINT_URL")
            if endpoint is None:
                raise OLMoEnvironmentError("Weka endpoint url is not set; did you forget WEKA_ENDPOINT_URL?")
            kwargs["endpoint_url"] = endpoint
        session = boto3.Session(profile_name=profile)
        client = session.client(
            "s3",
            config=Config(retries={"max_attempts": 10, "mode": "standard"}),
            use_ssl=not int(os.environ.get("OLMO_NO_SSL", "0")),
            **kwargs,
        )
        self._clients[scheme] = client
        return client

    @staticmethod
    def _split(url: str) -> Tuple[str, str, str]:
        u = urlparse(url)
        return u.scheme, u.netloc, u.path.strip("/")

    def file_size(self, url: str) -> int:
        scheme, bucket, key = self._split(url)

        def go() -> int:
            try:
                return self._client(scheme).head_object(Bucket=bucket, Key=key)["ContentLength"]
            except Exception as e:
                if getattr(e, "response", {}).get("ResponseMetadata", {}).get("HTTPStatusCode") == 404:
                    raise FileNotFoundError(url) from e
                raise

        return _retry(go, f"head {url}")

    def get_bytes_range(self, url: str, start: int, num: int) -> bytes:
        scheme, bucket, key = self._split(url)

        def go() -> bytes:
            try:
                obj = self._client(scheme).get_object(
                    Bucket=bucket, Key=key, Range=f"bytes={start}-{start + num - 1}"
                )
                return obj["Body"].read()
            except Exception as e:
                if getattr(e, "response", {}).get("ResponseMetadata", {}).get("HTTPStatusCode") == 404:
                    raise FileNotFoundError(url) from e
                raise

        return _retry(go, f"get {url}", max_attempts=4)

    def upload(self, source: Path, url: str, save_overwrite: bool = False) -> None:
        scheme, bucket, key = self._split(url)
        if not save_overwrite:
            try:
                self.file_size(url)
                raise FileExistsError(f"{url} already exists; use save_overwrite to replace it")
            except FileNotFoundError:
                pass
        _retry(lambda: self._client(scheme).upload_file(str(source), bucket, key), f"upload {url}")

    def find_latest_checkpoint(self, url: str) -> Optional[str]:
        scheme, bucket, prefix = self._split(url)
        if not prefix.endswith("/"):
            prefix += "/"
        resp = self._client(scheme).list_objects(Bucket=bucket, Prefix=prefix, Delimiter="/")
        assert not resp.get("IsTruncated", False)
        names = []
        for item in resp.get("CommonPrefixes", []):
            sub = item["Prefix"].strip("/")
            name = os.path.split(sub)[-1]
            if _STEP_DIR.match(name) is None:
                continue
            # a checkpoint counts only once its config.yaml has landed (it is uploaded last)
            try:
                self.file_size(f"{scheme}://{bucket}/{sub}/config.yaml")
            except FileNotFoundError:
                continue
            names.append(name)
        best = _pick_latest(names)
        return None if best is None else f"{scheme}://{bucket}/{prefix}{best}"

    def list_files(self, url: str) -> List[str]:
        scheme, bucket, prefix = self._split(url)
        if prefix and not prefix.endswith("/"):
            prefix += "/"
        out: List[str] = []
        token: Optional[str] = None
        while True:
            kwargs = {"Bucket": bucket, "Prefix": prefix}
            if token:
                kwargs["ContinuationToken"] = token
            resp = _retry(lambda: self._client(scheme).list_objects_v2(**kwargs), f"list {url}")
            out += [f"{scheme}://{bucket}/{item['Key']}" for item in resp.get("Contents", [])]
            token = resp.get("NextContinuationToken")
            if not token:
                return sorted(out)

    def delete(self, url: str) -> None:
        scheme, bucket, key = self._split(url)
        _retry(lambda: self._client(scheme).delete_object(Bucket=bucket, Key=key), f"delete {url}")


class _GcsBackend(StorageBackend):
    def _bucket(self, name: str):
        try:
            from google.cloud import storage as gcs
        except ImportError as e:
            raise OLMoEnvironmentError("'gs://' paths need the google-cloud-storage package") from e
        return gcs.Client().bucket(name)

    @staticmethod
    def _split(url: str) -> Tuple[str, str]:
        u = urlparse(url)
        return u.netloc, u.path.strip("/")

    def file_size(self, url: str) -> int:
        bucket, key = self._split(url)
        blob = self._bucket(bucket).blob(key)
        try:
            blob.reload()
        except Exception as e:
            if type(e).__name__ == "NotFound":
                raise FileNotFoundError(url) from e
            raise
        assert blob.size is not None
        return blob.size

    def get_bytes_range(self, url: str, start: int, num: int) -> bytes:
        bucket, key = self._split(url)
        blob = self._bucket(bucket).blob(key)
        return _retry(lambda: blob.download_as_bytes(start=start, end=start + num - 1), f"get {url}")

    def upload(self, source: Path, url: str, save_overwrite: bool = False) -> None:
        bucket, key = self._split(url)
        blob = self._bucket(bucket).blob(key)
        if not save_overwrite and blob.exists():
            raise FileExistsError(f"{url} already exists; use save_overwrite to replace it")
        _retry(lambda: blob.upload_from_filename(str(source)), f"upload {url}")

    def find_latest_checkpoint(self, url: str) -> Optional[str]:
        bucket, prefix = self._split(url)
        if not prefix.endswith("/"):
            prefix += "/"
        b = self._bucket(bucket)
        names = set()
        complete = set()
        for blob in b.list_blobs(prefix=prefix, match_glob=f"{prefix}step*/*"):
            rel = blob.name[len(prefix) :]
            d, _, f = rel.partition("/")
            names.add(d)
            if f == "config.yaml" and blob.size:
                complete.add(d)
        best = _pick_latest(n for n in names if n in complete)
        return None if best is None else f"gs://{bucket}/{prefix}{best}"

    def list_files(self, url: str) -> List[str]:
        bucket, prefix = self._split(url)
        if prefix and not prefix.endswith("/"):
            prefix += "/"
        return sorted(f"gs://{bucket}/{blob.name}" for blob in self._bucket(bucket).list_blobs(prefix=prefix))

    def delete(self, url: str) -> None:
        bucket, key = self._split(url)
        _retry(lambda: self._bucket(bucket).blob(key).delete(), f"delete {url}")


_BACKENDS: Dict[str, StorageBackend] = {}


def register_storage_backend(scheme: str, backend: StorageBackend) -> None:
    """Plug in (or replace, e.g. with a fake in tests) the handler of a URL scheme."""
    _BACKENDS[scheme] = backend


_local = _LocalBackend()
_s3 = _S3Backend()
register_storage_backend("", _local)
register_storage_backend("file", _local)
register_storage_backend("http", _HttpBackend())
register_storage_backend("https", _BACKENDS["http"])
for _scheme in ("s3", "r2", "weka"):
    register_storage_backend(_scheme, _s3)
register_storage_backend("gs", _GcsBackend())


def _backend_for(path: PathOrStr) -> Tuple[StorageBackend, str]:
    s = str(path)
    scheme = urlparse(s).scheme if is_url(s) else ""
    if scheme not in _BACKENDS:
        raise NotImplementedError(f"no storage back end for '{scheme}://' paths")
    return _BACKENDS[scheme], s


def file_size(path: PathOrStr) -> int:
    """Size in bytes of a local or remote file."""
    backend, s = _backend_for(path)
    return backend.file_size(s)


def get_bytes_range(source: PathOrStr, bytes_start: int, num_bytes: int) -> bytes:
    """Read ``num_bytes`` starting at ``bytes_start`` from a local or remote file."""
    backend, s = _backend_for(source)
    return backend.get_bytes_range(s, bytes_start, num_bytes)


def upload(source: PathOrStr, target: str, save_overwrite: bool = False) -> None:
    """Copy a local file to ``target`` (any scheme with an upload-capable back end)."""
    src = Path(source)
    if not src.is_file():
        raise FileNotFoundError(src)
    backend, s = _backend_for(target)
    backend.upload(src, s, save_overwrite=save_overwrite)


def find_latest_checkpoint(dir: PathOrStr) -> Optional[PathOrStr]:
    """Newest ``stepN[-unsharded]`` under ``dir``; a sharded checkpoint wins over an unsharded one
    of the same step (reference: ``olmo/util.py:393-419``)."""
    backend, s = _backend_for(dir)
    found = backend.find_latest_checkpoint(s)
    if found is None:
        return None
    return found if is_url(found) else Path(found)


def list_files(folder: PathOrStr) -> List[str]:
    """Every file below a local folder or remote prefix (full paths / URLs, sorted)."""
    backend, s = _backend_for(folder)
    return backend.list_files(s)


def delete_file(path: PathOrStr) -> None:
    """Remove one local or remote file."""
    backend, s = _backend_for(path)
    backend.delete(s)


def resource_path(
    folder: PathOrStr, fname: str, local_cache: Optional[PathOrStr] = None, progress: Any = None
) -> Path:
    """Return a local path for ``folder/fname``, downloading remote files into a cache directory."""
    if local_cache is not None and (cached := Path(local_cache) / fname).is_file():
        log.info("Found local cache of %s at %s", fname, cached)
        return cached
    full = f"{str(folder).rstrip('/')}/{fname}"
    if not is_url(full):
        p = Path(full)
        if not p.exists():
            raise FileNotFoundError(p)
        return p
    if full.startswith("file://"):
        return Path(full[len("file://") :])
    cache_root = Path(os.environ.get("OLMO_CACHE_DIR", Path.home() / ".cache" / "olmo_b200"))
    import hashlib

    target = cache_root / hashlib.sha256(full.encode()).hexdigest()[:16] / fname
    if not target.is_file():
        target.parent.mkdir(parents=True, exist_ok=True)
        size = file_size(full)
        tmp = target.with_suffix(target.suffix + ".part")
        with open(tmp, "wb") as f:
            chunk = 64 << 20
            for off in range(0, size, chunk):
                f.write(get_bytes_range(full, off, min(chunk, size - off)))
        os.replace(tmp, target)
    return target


def add_cached_path_clients() -> None:
    """Kept for entry-point parity: all schemes (``weka://`` included) are registered at import."""
    return None


# ---------------------------------------------------------------------------------------------
# Iterator tools
# ---------------------------------------------------------------------------------------------


def default_thread_count() -> int:
    return int(os.environ.get("OLMO_NUM_THREADS") or min(32, (os.cpu_count() or 1) + 4))


def pass_through_fn(fn, *args, **kwargs):
    return fn(*args, **kwargs)


def threaded_generator(g: Iterable[Any], maxsize: int = 16, thread_name: Optional[str] = None) -> Iterator[Any]:
    """Run generator ``g`` in a daemon thread and yield its items through a bounded queue.

    An exception in the producer surfaces in the consumer as :class:`OLMoThreadError`.
    """
    q: Queue = Queue(maxsize=maxsize)
    done = object()
    name = thread_name or repr(g)

    def produce() -> None:
        try:
            for item in g:
                q.put((None, item))
        except Exception as e:
            q.put((e, None))
        finally:
            q.put((None, done))

    Thread(name=name, target=produce, daemon=True).start()
    while True:
        err, item = q.get()
        if err is not None:
            raise OLMoThreadError(f"generator thread {name} failed") from err
        if item is done:
            return
        yield item


def roundrobin(*iterables: Iterable[Any]) -> Iterator[Any]:
    """``roundrobin('ABC', 'D', 'EF')`` yields ``A D E B F C``."""
    active = [iter(it) for it in iterables]
    while active:
        still = []
        for it in active:
            try:
                yield next(it)
                still.append(it)
            except StopIteration:
                pass
        active = still


def flatten_dict(dictionary, parent_key: str = "", separator: str = ".", include_lists: bool = False):
    """Nested mapping -> single-level mapping with ``separator``-joined keys."""
    flat: Dict[str, Any] = {}
    for key, value in dictionary.items():
        full = f"{parent_key}{separator}{key}" if parent_key else str(key)
        if include_lists and isinstance(value, list):
            value = {str(i): v for i, v in enumerate(value)}
        if isinstance(value, MutableMapping):
            flat.update(flatten_dict(value, full, separator=separator, include_lists=include_lists))
        else:
            flat[full] = value
    return flat


# ---------------------------------------------------------------------------------------------
# Packaged evaluation data (reference: olmo/util.py:730-802)
# ---------------------------------------------------------------------------------------------


def _data_roots() -> Iterable[Path]:
    env = os.environ.get("OLMO_DATA_DIR")
    if env:
        yield Path(env)
    yield Path(__file__).resolve().parent.parent / "olmo_data"
    try:
        import olmo_data  # the reference's data package, if it happens to be importable

        yield Path(olmo_data.__file__).resolve().parent
    except Exception:
        pass


def get_data_path(rel: str) -> Path:
    """Locate ``rel`` inside an ``olmo_data`` tree (``OLMO_DATA_DIR`` wins)."""
    for root in _data_roots():
        p = root / rel
        if p.exists():
            return p
    raise FileNotFoundError(f"'{rel}' not found in any olmo_data directory; set OLMO_DATA_DIR")


def load_hf_dataset(path: str, name: Optional[str], split: str):
    """Load a dataset that was stored with ``datasets.save_to_disk`` under ``hf_datasets/``."""
    import datasets

    rel = os.path.join("hf_datasets", path, name or "none", split)
    try:
        return datasets.load_from_disk(str(get_data_path(rel)))
    except FileNotFoundError as e:
        raise FileNotFoundError(f"HF dataset {path} name {name} split {split} not found under {rel}") from e


def save_hf_dataset_to_disk(dataset, hf_path: str, name: Optional[str], split: str, datasets_dir: PathOrStr) -> Path:
    """Store a ``datasets`` dataset where :func:`load_hf_dataset` looks for it: ``datasets_dir/<hf_path>/<name or "none">/<split>``
    (``datasets_dir`` is ``olmo_data/hf_datasets`` to add an evaluation set to the package data, or the ``hf_datasets`` folder
    of an ``OLMO_DATA_DIR`` tree).  Returns the folder."""
    target = Path(datasets_dir) / hf_path / (name or "none") / split
    target.parent.mkdir(parents=True, exist_ok=True)
    dataset.save_to_disk(str(target))
    return target


def load_oe_eval_requests(path: str, name: Optional[str] = None, split: Optional[str] = None):
    """Load an oe-eval request dump: returns ``(config_dict, [request, ...])``."""
    rel = os.path.join("oe_eval_tasks", path)
    if name is not None:
        rel = os.path.join(rel, name)
    root = get_data_path(rel)
    with open(root / "config.json") as f:
        config = json.load(f)
    split = split or config["task_config"]["split"]
    req_file = root / (f"{split}-requests.jsonl.gz" if (root / f"{split}-requests.jsonl.gz").exists() else "requests.jsonl.gz")
    with gzip.open(req_file, "rt") as f:
        requests = [json.loads(line) for line in f if line.strip()]
    return config, requests
