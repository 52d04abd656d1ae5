#!/usr/bin/env python
"""
Release helper with three sub-commands (the roles of the reference's ``scripts/prepare_changelog.py``,
``scripts/release_notes.py`` and ``scripts/release.sh``):

    python scripts/release.py stamp            # put the "Unreleased" entries of CHANGELOG.md under the package version
    python scripts/release.py notes [vX.Y.Z]   # print the notes of a version (default: the package version) + commits
    python scripts/release.py tag              # stamp, commit and create the git tag (asks first; pushes nothing)
"""
import argparse
import datetime
import re
import subprocess
import sys
from pathlib import Path
from typing import List, Optional

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

HEADERS = {"Added": "Added 🎉", "Changed": "Changed ⚠️", "Fixed": "Fixed ✅", "Removed": "Removed 👋"}


def package_version() -> str:
    from olmo_b200.version import VERSION

    return VERSION


def stamp(changelog: Path, version: str, today: Optional[str] = None) -> bool:
    """Insert a ``## [vX.Y.Z] - date`` heading right below ``## Unreleased``.  False when it is already there."""
    lines = changelog.read_text().splitlines(keepends=True)
    if any(line.startswith(f"## [v{version}]") for line in lines):
        return False
    try:
        at = next(i for i, line in enumerate(lines) if line.startswith("## Unreleased"))
    except StopIteration:
        raise RuntimeError("CHANGELOG.md has no 'Unreleased' section") from None
    today = today or datetime.date.today().isoformat()
    lines[at + 1 : at + 1] = ["\n", f"## [v{version}] - {today}\n"]
    changelog.write_text("".join(lines))
    return True


def notes(changelog: Path, tag: str) -> str:
    """The section of ``tag`` with decorated sub-headings."""
    out: List[str] = []
    inside = False
    for line in changelog.read_text().splitlines():
        if line.startswith("## "):
            if inside:
                break
            inside = line.startswith(f"## [{tag}]")
            continue
        if inside:
            m = re.match(r"### (\w+)\s*$", line)
            out.append(f"### {HEADERS.get(m.group(1), m.group(1))}" if m else line)
    if not any(l.strip() for l in out):
        raise RuntimeError(f"CHANGELOG.md has no entries for {tag}")
    return "## What's new\n\n" + "\n".join(out).strip() + "\n"


def _version_key(tag: str):
    parts = re.match(r"v(\d+)\.(\d+)\.(\d+)(.*)", tag)
    return (int(parts.group(1)), int(parts.group(2)), int(parts.group(3)), parts.group(4) == "", parts.group(4)) if parts else None


def commit_history(tag: str, cwd: Path = ROOT) -> str:
    """Commits since the latest earlier version tag (pre-releases are skipped unless ``tag`` is one)."""
    tags = subprocess.run(["git", "tag", "-l", "v*"], cwd=cwd, capture_output=True, text=True).stdout.split()
    mine = _version_key(tag)
    earlier = sorted((t for t in tags if _version_key(t) and mine and _version_key(t) < mine and (_version_key(t)[3] or not mine[3])), key=_version_key)
    span = f"{earlier[-1]}..HEAD" if earlier else "HEAD"
    log = subprocess.run(["git", "log", span, "--oneline", "--first-parent"], cwd=cwd, capture_output=True, text=True).stdout.strip()
    return "## Commits\n\n" + log + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = ap.add_subparsers(dest="command", required=True)
    sub.add_parser("stamp")
    p = sub.add_parser("notes")
    p.add_argument("tag", nargs="?")
    p.add_argument("--no-commits", action="store_true")
    sub.add_parser("tag")
    args = ap.parse_args(argv)
    changelog = ROOT / "CHANGELOG.md"
    version = package_version()
    if args.command == "stamp":
        print("CHANGELOG.md stamped" if stamp(changelog, version) else "CHANGELOG.md already up to date")
    elif args.command == "notes":
        tag = args.tag or f"v{version}"
        print(notes(changelog, tag) + ("" if args.no_commits else "\n" + commit_history(tag)))
    else:
        tag = f"v{version}"
        if input(f"Create release {tag}? [y/N] ").strip().lower() not in ("y", "yes"):
            print("cancelled")
            return 1
        stamp(changelog, version)
        subprocess.run(["git", "add", "CHANGELOG.md"], cwd=ROOT, check=True)
        subprocess.run(["git", "commit", "-m", f"Bump version to {tag} for release"], cwd=ROOT)
        subprocess.run(["git", "tag", tag, "-m", tag], cwd=ROOT, check=True)
        print(f"created tag {tag}; push with: git push && git push --tags")
    return 0


if __name__ == "__main__":
    sys.exit(main())
