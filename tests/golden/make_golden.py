"""Generate the golden fixtures that pin `oracle/kimi_oracle.py` to the reference implementation.

Run in a container where the reference (garv901/kimi-k3-goalbox) is importable:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference's own `megabench.tasks.kimi` (read-only), runs its BF16 and FP32 oracle on CPU
for a few small geometries and seeds, runs its band grader on perturbed candidates, and writes
`tests/golden/*.pt`. For every fixture it also stores a SHA-256 digest of each generated input tensor,
so the oracle restatement's seeded generator is pinned too. Two-rank fixtures run the reference with
torch.distributed over gloo on CPU. Nothing at run time (tests on a GPU box, bench, smoke) reads the
reference; they read only these files.
"""

from __future__ import annotations

import hashlib
import os
import sys
import tempfile
from dataclasses import replace
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent

# Geometry of the reference's own unit tests (megabench/tests/test_kimi.py:15-21): tiny dims.
TINY = {'layers': 5, 'hidden': 64, 'latent_hidden': 64, 'intermediate': 64, 'dense_intermediate': 128,
        'q_heads': 4, 'head_dim': 16, 'q_lora_rank': 32, 'kv_lora_rank': 32, 'qk_nope_dim': 8,
        'qk_rope_dim': 8, 'v_head_dim': 16, 'vocab': 128, 'experts': 8, 'topk': 2, 'context': 4,
        'attn_res_block_size': 2}

# The smallest geometry the CUDA kernels accept: Kimi's fixed head dims, small everything else.
SMALL = {'layers': 5, 'hidden': 256, 'latent_hidden': 128, 'intermediate': 128, 'dense_intermediate': 256,
         'q_heads': 2, 'head_dim': 128, 'q_lora_rank': 128, 'kv_lora_rank': 512, 'qk_nope_dim': 128,
         'qk_rope_dim': 64, 'v_head_dim': 128, 'vocab': 512, 'experts': 16, 'topk': 4, 'context': 16,
         'attn_res_block_size': 2}


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().view(torch.uint8).numpy().tobytes()).hexdigest()


def make_case(select_cases, base_id, params, batch, gpus=1):
    case = select_cases('all', [base_id])[0]
    return replace(case, params=case.params | params | {'batch': batch}, gpus=gpus, tp=gpus)


def serial_fixture(kimi, case, seed):
    values = kimi.make_inputs(case, seed, 'cpu', rank=0)
    bf16 = kimi.reference(case, values, serial=True)
    fp32 = kimi.reference(case, values, serial=True, fp32=True)
    forced = kimi.reference(case, values, serial=True, fp32=True, routes=bf16['expert_ids'])
    # band-grader pins: the oracle itself, FP32 cast to the output dtypes, noisy logits, flipped routes
    gen = torch.Generator().manual_seed(seed)
    noisy = dict(bf16, logits=bf16['logits'] + 0.05 * bf16['logits'].std() * torch.randn(bf16['logits'].shape, generator=gen))
    as_fp32 = {k: (fp32[k].to(v.dtype) if k not in ('expert_ids', 'next_token') else v) for k, v in bf16.items()}
    grades = {}
    for label, cand in (('oracle', {k: v.clone() for k, v in bf16.items()}), ('fp32', as_fp32),
                        ('noisy', noisy), ('flipped', dict(bf16, expert_ids=bf16['expert_ids'].flip(-1)))):
        try:
            grades[label] = {'ok': True, 'details': kimi.compare(case, values, bf16, cand, serial=True)}
        except AssertionError as exc:
            grades[label] = {'ok': False, 'error': str(exc)}
    # the FP32 recurrent state is the bulk of a fixture: keep its digest and a strided sample
    state = fp32.pop('recurrent_state')
    fp32['recurrent_state_digest'] = digest(state)
    fp32['recurrent_state_sample'] = state.flatten()[::97].clone()
    return {'case': case.to_dict(), 'seed': seed, 'inputs': {k: digest(v) for k, v in values.items()},
            'bf16': bf16, 'fp32': fp32, 'forced_shortfall': forced['route_shortfall'],
            'noisy_logits': noisy['logits'], 'grades': grades}


def _tp_worker(rank, world, ref_root, case_dict, seed, out_dir, init):
    sys.path.insert(0, ref_root)
    import torch.distributed as dist
    from megabench.cases import Case
    from megabench.tasks import kimi
    dist.init_process_group('gloo', init_method=init, rank=rank, world_size=world)
    try:
        case = Case(**case_dict)
        values = kimi.make_inputs(case, seed, 'cpu')
        out = kimi.reference(case, values)
        grade = kimi.compare(case, values, out, {k: v.clone() for k, v in out.items()})
        torch.save({'inputs': {k: digest(v) for k, v in values.items()}, 'bf16': out, 'grade': grade},
                   os.path.join(out_dir, f'rank{rank}.pt'))
    finally:
        dist.destroy_process_group()


def tp_fixture(case, seed, ref_root):
    import torch.multiprocessing as mp
    with tempfile.TemporaryDirectory() as tmp:
        init = (Path(tmp) / 'rdv').as_uri()
        mp.spawn(_tp_worker, nprocs=case.gpus, args=(case.gpus, ref_root, case.to_dict(), seed, tmp, init))
        ranks = [torch.load(os.path.join(tmp, f'rank{r}.pt')) for r in range(case.gpus)]
    return {'case': case.to_dict(), 'seed': seed, 'ranks': ranks}


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from megabench.cases import select_cases
    from megabench.tasks import kimi
    torch.set_num_threads(4)
    dev = 'kimi-k3-dev-l4-tp1-b8-s8192'
    fixtures = {
        'tiny_b3_s21': serial_fixture(kimi, make_case(select_cases, dev, TINY, 3), 21),
        'tiny_b1_s9': serial_fixture(kimi, make_case(select_cases, dev, TINY, 1), 9),   # seed % 3 == 0: B=1 reset
        'small_b3_s7': serial_fixture(kimi, make_case(select_cases, dev, SMALL, 3), 7),
    }
    for name, fx in fixtures.items():
        torch.save(fx, HERE / f'{name}.pt')
    tp2 = tp_fixture(make_case(select_cases, dev, TINY, 2, gpus=2), 5, ref_root)
    torch.save(tp2, HERE / 'tiny_tp2_b2_s5.pt')
    # the reference's HBM floor model (megabench/sol.py) on every case of its table
    import json
    from megabench.sol import estimate_case
    sol = {c.id: {'minimum_bytes': estimate_case(c)['minimum_bytes'],
                  'components': {x['name']: x['bytes'] for x in estimate_case(c)['components']}}
           for c in select_cases('all')}
    (HERE / 'sol_reference.json').write_text(json.dumps(sol, indent=1) + '\n')
    for path in sorted(HERE.glob('*.pt')):
        print(path.name, path.stat().st_size)


if __name__ == '__main__':
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py /path/to/reference")
    main(sys.argv[1])
