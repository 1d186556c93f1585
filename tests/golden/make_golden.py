"""Writes tests/golden/sampler_kats.json: hand-derived known answers for the
reference's two samplers (src/snai_inference.php:151-195 = variant 0,
src/tensor_ffi_adapter.php:168-204 = variant 1).

The reference ships no golden vectors and cannot run here (no PHP), so every
expected id below is derived by hand from the PHP source; the derivation is
in the comment beside each case.  Nothing here is computed by the oracle.

Run:  python tests/golden/make_golden.py
"""
import json
import os

INF = "-inf"  # JSON has no infinities; the loader maps this string back

CASES = [
    # ---------------- variant 0 (inference script) ----------------
    dict(name="A_u0_returns_0", variant=0, logits=[0.5, 3.0, 1.0, -2.0], hist=[], T=0.8, rep=1.15, u=0.0,
         expect=0, why="r = 0*sum = 0 and cumulative = p_0 >= 0 at v = 0 (:186-193)"),
    dict(name="A_greedy_all_equal", variant=0, logits=[1.0] * 8, hist=[], T=0.01, rep=1.15, u=0.5,
         expect=0, why="T <= 0.01 is greedy; strict > keeps the first maximum (:170-172)"),
    dict(name="A_greedy_spike", variant=0, logits=[0.0] * 5 + [10.0] + [0.0] * 4, hist=[], T=0.01, rep=1.0, u=0.5,
         expect=5, why="the spike is the unique maximum"),
    dict(name="A_greedy_tie_lowest", variant=0, logits=[1.0, 3.0, 3.0, 2.0], hist=[], T=0.01, rep=1.0, u=0.5,
         expect=1, why="ties keep the lowest index (:170)"),
    dict(name="A_uniform_draw", variant=0, logits=[0.0, 0.0, 0.0, 0.0], hist=[], T=1.0, rep=1.0, u=0.6,
         expect=2, why="p = 1 each, sum 4, r = 2.4; running sums 1, 2, 3 -> first >= 2.4 is v = 2"),
    dict(name="A_penalty_positive", variant=0, logits=[2.0, 1.5], hist=[0], T=0.01, rep=2.0, u=0.5,
         expect=1, why="200 > 0 -> 200/2 = 100 < 150 (:160-161)"),
    dict(name="A_penalty_negative", variant=0, logits=[-1.0, -1.5], hist=[0], T=0.01, rep=2.0, u=0.5,
         expect=1, why="-100 <= 0 -> -100*2 = -200 < -150 (:162-163)"),
    dict(name="A_penalty_once_per_id", variant=0, logits=[2.0, 1.5], hist=[0, 0, 0], T=0.01, rep=1.2, u=0.5,
         expect=0, why="array_unique: 200/1.2 = 166.7 > 150 (three times would give 115.7 < 150)"),
    dict(name="A_u1_last_nonzero", variant=0, logits=[0.0, 0.0, -1000.0], hist=[], T=1.0, rep=1.0, u=1.0,
         expect=1, why="p = 1, 1, exp(-1000) = 0; r = sum = 2 reached at v = 1"),
    dict(name="A_history_out_of_range_ignored", variant=0, logits=[2.0, 1.5], hist=[7, -3], T=0.01, rep=4.0,
         u=0.5, expect=0, why="ids outside [0,V) touch no logit"),
    # ---------------- variant 1 (bridge generate_next_token) ----------------
    dict(name="B_topk1_is_argmax", variant=1, logits=[1.0, 3.0, 3.0, 2.0], hist=[], T=0.7, top_k=1, top_p=0.9,
         rep=1.15, u=0.73, expect=1,
         why="stable arsort puts id 1 before id 2; one survivor, r <= its cum (:177-204)"),
    dict(name="B_topp_tiny_is_top1", variant=1, logits=[0.0, 5.0, 1.0, 2.0], hist=[], T=1.0, top_k=3, top_p=1e-9,
         rep=1.0, u=0.99, expect=1, why="the first p_norm already reaches top_p (:194)"),
    dict(name="B_greedy_tie_lowest", variant=1, logits=[2.0, 7.0, 7.0], hist=[], T=0.0, top_k=3, top_p=0.9,
         rep=1.0, u=0.5, expect=1, why="T < 0.01 returns the first key of the stable descending order (:180)"),
    dict(name="B_penalty_subtracts", variant=1, logits=[3.0, 2.5], hist=[0], T=0.001, top_k=2, top_p=0.9,
         rep=1.0, u=0.5, expect=1, why="3 - 1 = 2 < 2.5 (:171-175), then greedy"),
    dict(name="B_u0_first_sorted", variant=1, logits=[1.0, 4.0, 2.0], hist=[], T=1.0, top_k=3, top_p=1.0, rep=1.0,
         u=0.0, expect=1, why="r = 0 <= the first running sum; order is 1, 2, 0"),
    dict(name="B_draw_first", variant=1, logits=[0.0, 1.0986122886681098], hist=[], T=1.0, top_k=2, top_p=1.0,
         rep=1.0, u=0.5, expect=1, why="p = 3:1 -> 0.75, 0.25 in order (1, 0); r = 0.5 <= 0.75"),
    dict(name="B_draw_second", variant=1, logits=[0.0, 1.0986122886681098], hist=[], T=1.0, top_k=2, top_p=1.0,
         rep=1.0, u=0.9, expect=0, why="r = 0.9 > 0.75, <= 1.0 at the second id (0)"),
    dict(name="B_equal_logits_index_order", variant=1, logits=[0.5] * 100, hist=[], T=1.0, top_k=5, top_p=1.0,
         rep=1.0, u=0.99, expect=4,
         why="ties keep index order: survivors 0..4 with 0.2 each; r = 0.99 <= 1.0 only at the 5th (id 4)"),
    dict(name="B_topp_cut_includes_crossing", variant=1, logits=[0.0, 1.0986122886681098], hist=[], T=1.0,
         top_k=2, top_p=0.5, rep=1.0, u=0.99, expect=1,
         why="cum 0.75 >= 0.5 stops after id 1 (crossing included); r = 0.99*0.75 <= 0.75"),
]


def main():
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampler_kats.json")
    with open(out, "w") as f:
        json.dump({"source": "hand-derived from the PHP samplers; see make_golden.py", "cases": CASES}, f,
                  indent=1)
    print(f"wrote {len(CASES)} cases to {out}")


if __name__ == "__main__":
    main()
