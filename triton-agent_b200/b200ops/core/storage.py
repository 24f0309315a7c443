"""Episode and leaderboard storage (interfaces of triton_agent/core/storage.py:12-165).

EpisodeStore writes one JSON record per evaluated candidate under
<dir>/<op>/<episode_id>/record.json (storage.py:12-65).  LeaderboardStore keeps
the best configuration per (op, shape, dtype, device, template) in SQLite
(storage.py:68-165) with the CUDA launch parameters this backend tunes
(threads, rows_per_cta, split, tile_m/n/k, flags, stages) and the roofline fields of
the measurement (achieved GB/s or TOPS, roofline fraction) instead of the
reference's Triton block/warp columns only.  Together with
microrl.trainer.ShapeConfigStore they let a later tuning run start from the
best known configuration.
"""

from __future__ import annotations

import json
import sqlite3
import time
from contextlib import contextmanager
from pathlib import Path
from typing import Any, Iterator

from .spec import CandidateResult, OpAction, OpState


class EpisodeStore:
    def __init__(self, episodes_dir: str | Path = "episodes") -> None:
        self.episodes_dir = Path(episodes_dir)
        self.episodes_dir.mkdir(parents=True, exist_ok=True)

    def save(self, op_name: str, episode_id: str, state: OpState, action: OpAction, result: CandidateResult,
             extra: dict[str, Any] | None = None) -> Path:
        d = self.episodes_dir / op_name / episode_id
        d.mkdir(parents=True, exist_ok=True)
        record = {"episode_id": episode_id, "timestamp": time.time(), "state": state.to_dict(),
                  "action": action.to_dict(), "result": result.to_dict(), "extra": extra or {}}
        (d / "record.json").write_text(json.dumps(record, indent=2, default=str))
        return d

    def load(self, op_name: str, episode_id: str) -> dict | None:
        p = self.episodes_dir / op_name / episode_id / "record.json"
        return json.loads(p.read_text()) if p.exists() else None

    def list_episodes(self, op_name: str) -> list[str]:
        d = self.episodes_dir / op_name
        if not d.exists():
            return []
        return sorted(e.name for e in d.iterdir() if (e / "record.json").exists())


_COLUMNS = (
    ("op_name", "TEXT NOT NULL"), ("shape", "TEXT NOT NULL"), ("dtype", "TEXT NOT NULL"),
    ("device", "TEXT NOT NULL"), ("template_id", "TEXT"),
    ("block_d", "INTEGER"), ("num_warps", "INTEGER"), ("num_stages", "INTEGER"), ("vectorize", "INTEGER"),
    ("threads", "INTEGER"), ("rows_per_cta", "INTEGER"), ("split", "INTEGER"), ("tile_m", "INTEGER"),
    ("tile_n", "INTEGER"), ("tile_k", "INTEGER"), ("flags", "INTEGER"),
    ("latency_us_p50", "REAL"), ("speedup", "REAL"), ("reward", "REAL"), ("promoted", "INTEGER"),
    ("achieved_GBps", "REAL"), ("achieved_TOPS", "REAL"), ("roofline_fraction", "REAL"), ("num_gpus", "INTEGER"),
    ("episode_id", "TEXT"), ("timestamp", "REAL"),
)
_KEY = ("op_name", "shape", "dtype", "device", "template_id")


class LeaderboardStore:
    def __init__(self, db_path: str | Path = "leaderboard/leaderboard.sqlite") -> None:
        self.db_path = Path(db_path)
        self.db_path.parent.mkdir(parents=True, exist_ok=True)
        cols = ",\n".join(f"{n} {t}" for n, t in _COLUMNS)
        with self._conn() as conn:
            conn.execute(f"CREATE TABLE IF NOT EXISTS leaderboard (id INTEGER PRIMARY KEY AUTOINCREMENT, {cols}, "
                         f"UNIQUE({', '.join(_KEY)}))")
            # a table written before a column existed gains it (NULL in old rows)
            have = {r[1] for r in conn.execute("PRAGMA table_info(leaderboard)")}
            for n, t in _COLUMNS:
                if n not in have:
                    conn.execute(f"ALTER TABLE leaderboard ADD COLUMN {n} {t.replace(' NOT NULL', '')}")

    @contextmanager
    def _conn(self) -> Iterator[sqlite3.Connection]:
        """One connection per operation: committed on success, rolled back on
        error, closed either way."""
        conn = sqlite3.connect(str(self.db_path))
        try:
            with conn:
                yield conn
        finally:
            conn.close()

    def upsert(self, op_name: str, shape: str, dtype: str, device: str, action: OpAction, result: CandidateResult,
               episode_id: str) -> None:
        """Inserts the row; a row with the same (op, shape, dtype, device,
        template) key is overwritten by the newer measurement (storage.py:102-137)."""
        row = {"op_name": op_name, "shape": shape, "dtype": dtype, "device": device,
               "template_id": action.template_id, "block_d": action.block_d, "num_warps": action.num_warps,
               "num_stages": action.num_stages, "vectorize": int(bool(action.vectorize)),
               "threads": action.threads, "rows_per_cta": action.rows_per_cta, "split": action.split,
               "tile_m": action.tile_m, "tile_n": action.tile_n, "tile_k": action.tile_k, "flags": action.flags,
               "latency_us_p50": result.latency_us_p50, "speedup": result.speedup, "reward": result.reward,
               "promoted": int(bool(result.promoted)), "achieved_GBps": result.achieved_GBps,
               "achieved_TOPS": result.achieved_TOPS, "roofline_fraction": result.roofline_fraction,
               "num_gpus": result.num_gpus, "episode_id": episode_id, "timestamp": time.time()}
        names = [n for n, _ in _COLUMNS]
        updates = ", ".join(f"{n}=excluded.{n}" for n in names if n not in _KEY)
        sql = (f"INSERT INTO leaderboard ({', '.join(names)}) VALUES ({', '.join('?' for _ in names)}) "
               f"ON CONFLICT({', '.join(_KEY)}) DO UPDATE SET {updates}")
        with self._conn() as conn:
            conn.execute(sql, [row[n] for n in names])

    def query(self, op_name: str, shape: str | None = None, dtype: str | None = None, limit: int = 20) -> list[dict]:
        where, params = ["op_name = ?"], [op_name]
        if shape:
            where.append("shape = ?")
            params.append(shape)
        if dtype:
            where.append("dtype = ?")
            params.append(dtype)
        with self._conn() as conn:
            conn.row_factory = sqlite3.Row
            rows = conn.execute(f"SELECT * FROM leaderboard WHERE {' AND '.join(where)} "
                                f"ORDER BY speedup DESC LIMIT ?", params + [limit]).fetchall()
        return [dict(r) for r in rows]

    def best_config(self, op_name: str, shape: str, dtype: str) -> dict | None:
        rows = self.query(op_name, shape=shape, dtype=dtype, limit=1)
        return rows[0] if rows else None

    @staticmethod
    def action_of(row: dict) -> OpAction:
        """The OpAction a leaderboard row was measured with (to re-run or warm start)."""
        return OpAction(template_id=row["template_id"], block_d=row["block_d"], num_warps=row["num_warps"],
                        num_stages=row["num_stages"], vectorize=bool(row["vectorize"]), threads=row["threads"],
                        rows_per_cta=row["rows_per_cta"], split=row["split"], tile_m=row["tile_m"],
                        tile_n=row["tile_n"], tile_k=row["tile_k"], flags=row.get("flags") or 0)
