"""Generate the small challenge-bank JSONL fixtures used by the bank tests.

Runs the reference's own bank generator (challenge_bank.py: build_records,
challenge_bank.py:346-397) from a reference checkout, at a few levels per
split and family, and writes its records exactly as its CLI does
(challenge_bank.py:427-429). The CLI's "at least 30 per split" rule only keeps
difficulty bands balanced at scale, so build_records is called directly.

    python tests/golden/make_challenge_bank.py --reference <checkout>
"""
import argparse
import hashlib
import importlib.util
import json
import pathlib

HERE = pathlib.Path(__file__).resolve().parent


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", type=pathlib.Path, required=True)
    args = parser.parse_args()
    spec = importlib.util.spec_from_file_location("challenge_bank", args.reference / "challenge_bank.py")
    bank = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bank)
    world_hash = hashlib.sha256((args.reference / "world.hpp").read_bytes()).hexdigest()
    for name, per_split, mirror in (("challenge_bank_small.jsonl", 4, False),
                                    ("challenge_bank_mirrored_small.jsonl", 4, True)):
        records = bank.build_records(20261001, per_split, 8.0, [14, 15, 16], world_hash, mirror)
        with (HERE / name).open("w", encoding="utf-8") as out:
            for record in records:
                out.write(json.dumps(record, sort_keys=True, separators=(",", ":")) + "\n")
        print(f"wrote {name}: {len(records)} records, world hash {world_hash}")


if __name__ == "__main__":
    main()
