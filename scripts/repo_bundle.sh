#!/usr/bin/env bash
# Pack the working tree (tracked + untracked-but-not-ignored files, never .git) into a tar.gz, or
# unpack such an archive into a fresh directory beside the repo.  The built extension (*.so) is
# ignored by git and therefore not packed: rebuild it on the target with `python setup.py build_ext --inplace`.
#
#   scripts/repo_bundle.sh pack [archive.tar.gz]      (default: <repo>_<UTC timestamp>.tar.gz in the parent dir)
#   scripts/repo_bundle.sh unpack <archive.tar.gz> [dest_dir]
set -Eeuo pipefail

die() { echo "Error: $*" >&2; exit 1; }

usage() { sed -n '2,8p' "$0" | sed 's/^# \{0,1\}//'; }

here="$(cd -- "$(dirname -- "${BASH_SOURCE[0]}")" && pwd -P)"
repo="$(cd -- "$here/.." && pwd -P)"
name="$(basename -- "$repo")"

pack() {
  git -C "$repo" rev-parse --is-inside-work-tree >/dev/null 2>&1 || die "not inside a git work tree: $repo"
  local out="${1:-$(dirname -- "$repo")/${name}_$(date -u +%Y%m%dT%H%M%SZ).tar.gz}"
  [[ "$out" = /* ]] || out="$PWD/$out"
  local list
  list="$(mktemp)"
  trap 'rm -f "$list"' RETURN
  git -C "$repo" ls-files --cached --others --exclude-standard -z > "$list"
  [[ -s "$list" ]] || die "nothing to pack"
  tar -C "$repo" --null -T "$list" --ignore-failed-read -czf "$out"
  echo "packed $(tr -cd '\0' < "$list" | wc -c) files into $out"
}

unpack() {
  local archive="${1:-}"
  [[ -n "$archive" ]] || die "unpack needs an archive path"
  [[ -f "$archive" ]] || archive="$repo/$archive"
  [[ -f "$archive" ]] || die "archive not found: $1"
  local base dest
  base="$(basename -- "$archive" .tar.gz)"
  dest="${2:-$(dirname -- "$repo")/$base}"
  [[ -e "$dest" ]] && die "destination exists: $dest"
  mkdir -p "$dest"
  tar -C "$dest" -xzf "$archive"
  echo "unpacked into $dest"
}

case "${1:-}" in
  pack) shift; pack "$@" ;;
  unpack) shift; unpack "$@" ;;
  -h|--help|help|"") usage ;;
  *) usage; die "unknown command: $1" ;;
esac
