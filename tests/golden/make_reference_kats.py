"""Writes tests/golden/reference_kats.json: the known-answer tests of the
reference's own test blocks for this path, transcribed as data.

The reference (Zig) cannot be built or run here, so its test assertions are the
golden vectors: each case lists the operations of one reference `test` block and
the values it asserts, with the source file:line.  Run:
    python tests/golden/make_reference_kats.py
"""
import json
from pathlib import Path

RING = [
    {"name": "ring buffer tiers and window eviction", "src": "src/ring_buffer.zig:393-410",
     "init": [2, 4], "ops": [["writeKV", 0, c] for c in range(20)],
     "checks": [["active_count", 0, 19, False, 1024, 20], ["active_at", 0, 19, False, 1024, 0, 0],
                ["active_at", 0, 19, False, 1024, 3, 3]]},
    {"name": "recall slots are written, cleared, and included in active set", "src": "src/ring_buffer.zig:412-431",
     "init": [32, 2], "ops": [["writeRecallKV", 16, 0, 100], ["writeRecallKV", 16, 1, 50]],
     "checks": [["active_count", 16, 101, False, 1024, 2]],
     "then": {"ops": [["clearRecall"]], "checks": [["active_count", 16, 101, False, 1024, 0]]}},
    {"name": "prefill slot calculation strictly respects physical ring buffer bounds", "src": "src/ring_buffer.zig:433-468",
     "init": [2, 512], "ops": [["activate_write", 0, 5000]],
     "checks": [["prefill_prev_bounds", 0, 5000, 226, 512]]},
    {"name": "ring buffer rollbackClock cleanly deactivates transient probe slots", "src": "src/ring_buffer.zig:575-597",
     "init": [2, 4], "ops": [["activate_range", 0, 10, 2]],
     "checks": [["total_ingested", 10]],
     "then": {"ops": [["activate_range", 10, 13, 2]], "checks": [["total_ingested", 13], ["slot_active_of_clock", 0, 11, True]],
              "then": {"ops": [["rollbackClock", 10]],
                       "checks": [["total_ingested", 10], ["slot_active_of_clock", 0, 11, False]]}}},
]

# salience / Gini / eviction tests exercise oracle-only metadata (not on the decode path)
RING_ORACLE_ONLY = [
    {"name": "attention mass accumulation and salience scoring", "src": "src/ring_buffer.zig:470-486",
     "init": [4, 4], "ops": [["activate", l, 0] for l in range(4)] +
     [["recordAttention", 0, 0, 0.5], ["recordAttention", 1, 0, 0.7], ["recordAttention", 2, 0, 0.4],
      ["recordAttention", 3, 0, 0.8]],
     "checks": [["mass_eq", 0, 0, 0.5], ["salience_eq", 0, 0.6]]},
    {"name": "evictLowSalienceSlots evicts low salience tokens and preserves heavy hitters",
     "src": "src/ring_buffer.zig:488-528", "init": [2, 4],
     "ops": [["writeKV", l, c] for c in range(4, 10) for l in (0, 1)] +
     [["recordAttentionClock", 0, 6, 10.0], ["recordAttentionClock", 1, 6, 10.0]] +
     [["recordAttentionClock", l, c, 1.0] for c in range(7, 10) for l in (0, 1)] +
     [["recordAttentionClock", 0, 4, 0.1], ["recordAttentionClock", 0, 5, 0.2]],
     "checks": [["evict", 4, 9, 2, 2], ["slot_active_of_clock", 0, 4, False], ["slot_active_of_clock", 0, 5, False],
                ["slot_active_of_clock", 0, 6, True]]},
    {"name": "getWorkingSetGini distinguishes focused vs diffuse attention distributions (flat)",
     "src": "src/ring_buffer.zig:530-551", "init": [2, 4],
     "ops": [["writeKV", 0, c] for c in range(4, 8)] + [["recordAttentionClock", 0, c, 1.0] for c in range(4, 8)],
     "checks": [["gini_lt", 0.10], ["saturated", 0.0005, 0.35, True]]},
    {"name": "getWorkingSetGini distinguishes focused vs diffuse attention distributions (skewed)",
     "src": "src/ring_buffer.zig:553-572", "init": [2, 4],
     "ops": [["writeKV", 0, c] for c in range(4, 8)] +
     [["recordAttentionClock", 0, 4, 0.05], ["recordAttentionClock", 0, 5, 0.05], ["recordAttentionClock", 0, 6, 0.10],
      ["recordAttentionClock", 0, 7, 10.0]],
     "checks": [["gini_gt", 0.60], ["saturated", 0.0005, 0.35, False]]},
]

SAMPLER = [
    {"name": "sampler.sampleTopK re-sorts penalized candidates (greedy half)", "src": "src/sampler.zig:429-446",
     "cands": [[4373, 18.0], [705, 17.5], [1980, 16.0]], "recent": [4373, 4373],
     "repeat": 1.2, "freq": 0.1, "pres": 0.1, "think": 0, "close": 0, "crit": 0, "expect": 705},
    {"name": "sampler.sampleTopK frequency and presence penalties suppress repeated tokens",
     "src": "src/sampler.zig:455-473", "cands": [[6639, 18.0], [16132, 17.0]], "recent": [6639, 6639, 6639],
     "repeat": 1.0, "freq": 0.5, "pres": 0.5, "think": 0, "close": 0, "crit": 0, "expect": 16132},
    {"name": "sampler.sampleTopK suppresses token 100 when suppress_thinking is active", "src": "src/sampler.zig:475-486",
     "cands": [[100, 20.0], [236777, 15.0]], "recent": None,
     "repeat": 1.1, "freq": 0.1, "pres": 0.1, "think": 1, "close": 0, "crit": 0, "expect": 236777},
    {"name": "sampler.sampleTopK suppresses token 101 when suppress_channel_close is active",
     "src": "src/sampler.zig:488-499", "cands": [[101, 25.0], [120474, 20.0]], "recent": None,
     "repeat": 1.1, "freq": 0.1, "pres": 0.1, "think": 0, "close": 1, "crit": 0, "expect": 120474},
    {"name": "sampler.sampleTopK suppresses critique tokens when suppress_critique is active",
     "src": "src/sampler.zig:501-515", "cands": [[20470, 22.0], [68755, 21.0], [4573, 20.0], [705, 15.0]],
     "recent": None, "repeat": 1.1, "freq": 0.1, "pres": 0.1, "think": 0, "close": 0, "crit": 1, "expect": 705},
]

BF16 = {"name": "bfloat16 roundtrip", "src": "src/tensor.zig:30-41",
        "cases": [[3.1415926, 0.02], [0.0, 0.0], [-42.5, 0.1]]}

if __name__ == "__main__":
    out = Path(__file__).with_name("reference_kats.json")
    out.write_text(json.dumps({"ring": RING, "ring_oracle_only": RING_ORACLE_ONLY, "sampler": SAMPLER, "bf16": BF16},
                              indent=1) + "\n")
    print(out)
