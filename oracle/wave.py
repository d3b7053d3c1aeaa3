"""Wave-quantisation analysis oracle (pure Python, no GPU).

Restates the reference's analytic model:
* ceil_div, wave_efficiency        sm_aware_matmul.py:17-28
* CONFIGS (candidate tile list)    sm_aware_matmul.py:31-48
* rank_configs (best per SM level) sm_aware_matmul.py:60-67  (sort key (waves, -last_util))
* compute_wave_efficiency          sm_aware_agent/workload.py:86-107
* suggest_optimal_block_size       sm_aware_agent/workload.py:110-143
"""
from __future__ import annotations

# Candidate (BLOCK_SIZE_M, BLOCK_SIZE_N, BLOCK_SIZE_K) list of the reference's
# analytical mode, in its order (order matters: the ranking sort is stable).
CONFIGS = [
    (128, 256, 64), (64, 256, 32), (128, 128, 32), (128, 64, 32), (64, 128, 32), (128, 32, 32), (64, 32, 32),
    (32, 64, 32), (128, 256, 128), (256, 128, 128), (256, 64, 128), (64, 256, 128), (128, 128, 128),
    (128, 64, 64), (64, 128, 64), (128, 32, 64),
]

# Default (BLOCK_M, BLOCK_N) candidates of suggest_optimal_block_size, in order.
SUGGEST_BLOCKS = [(16, 64), (32, 64), (32, 128), (64, 64), (64, 128), (128, 64), (128, 128), (128, 256),
                  (256, 128), (64, 256), (256, 64)]


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def wave_efficiency(M: int, N: int, bm: int, bn: int, num_sms: int) -> tuple[int, float, float]:
    """(waves, last-wave utilisation, overall efficiency) of a one-tile-per-CTA grid."""
    blocks = ceil_div(M, bm) * ceil_div(N, bn)
    waves = ceil_div(blocks, num_sms)
    last = blocks % num_sms
    if last == 0:
        last = num_sms
    return waves, last / num_sms, blocks / (waves * num_sms)


def rank_configs(M: int, N: int, num_sms: int, configs=CONFIGS) -> list[tuple]:
    """Configs ranked as the reference's analytical mode does: fewest waves,
    then fullest last wave; ties keep list order."""
    ranked = []
    for c in configs:
        nw, lwu, eff = wave_efficiency(M, N, c[0], c[1], num_sms)
        ranked.append((c, nw, lwu, eff))
    ranked.sort(key=lambda x: (x[1], -x[2]))
    return ranked


def compute_wave_efficiency(M: int, N: int, bm: int, bn: int, num_sms: int) -> dict:
    blocks = ((M + bm - 1) // bm) * ((N + bn - 1) // bn)
    waves = (blocks + num_sms - 1) // num_sms
    last = blocks % num_sms
    if last == 0:
        last = num_sms
    return {
        "num_blocks": blocks,
        "num_waves": waves,
        "last_wave_util": last / num_sms,
        "overall_efficiency": blocks / (waves * num_sms) if waves > 0 else 0,
    }


def suggest_optimal_block_size(M: int, N: int, num_sms: int, block_sizes=None):
    """First candidate with strictly the highest overall efficiency."""
    if block_sizes is None:
        block_sizes = SUGGEST_BLOCKS
    best = None
    best_eff = 0
    for bm, bn in block_sizes:
        m = compute_wave_efficiency(M, N, bm, bn, num_sms)
        if m["overall_efficiency"] > best_eff:
            best_eff = m["overall_efficiency"]
            best = (bm, bn, m)
    return best
