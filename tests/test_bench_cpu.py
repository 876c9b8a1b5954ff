"""Host logic of bench.py that needs no GPU: both arms report one workload config."""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import bench  # noqa: E402


def _args(streams=64, backbone='shared'):
    return argparse.Namespace(group=8, prompt=512, streams=streams, lanes=8, backbone=backbone, step_table=1, ln12=0)


def test_frame_config_keys_and_backbone_mode():
    a = _args()
    c = bench.frame_config(a, 2, 64, 8, True, 18, [513, 540])
    assert c['streams'] == 128 and c['streams_per_gpu'] == 64 and c['parallelism'] == 'replica x2'
    assert c['backbone'] == 'shared' and 'row groups of 64' in c['workload']
    assert set(c) >= {'workload', 'streams', 'streams_per_gpu', 'step', 'streams_per_launch', 'prompt_len',
                      'kv_len', 'parallelism', 'lanes', 'backbone', 'lane_sms', 'l2', 'cb0', 'prefill'}
    c2 = bench.frame_config(a, 1, 128, 8, False, 18, [513, 540])
    assert c2['backbone'] == 'lanes' and 'a backbone graph per 8 streams' in c2['workload']


def test_reference_arm_describes_its_own_work():
    """The reference arm's config says what it runs: one stream of the CPU port with the reference server's cache
    capacity and the host's thread count -- not the GPU arm's multi-stream workload."""
    a = _args()
    c = bench.reference_config(a, 7)
    assert c['streams'] == 1 and c['device'] == 'cpu' and c['threads'] == 7
    assert c['cache_len'] == bench.CPU_CACHE_LEN == 2048 and c['prompt_len'] == 512
    assert 'lanes' not in c and 'streams_per_gpu' not in c


def test_cpu_threads_ignore_omp_num_threads(monkeypatch):
    """Both CPU legs size their BLAS pool from the process's CPU affinity, not from OMP_NUM_THREADS (torchrun sets
    it to 1)."""
    monkeypatch.setenv('OMP_NUM_THREADS', '1')
    assert bench.cpu_threads() == len(os.sched_getaffinity(0))


def test_cpu_frames_one_frame_small_cache():
    """The shared CPU leg runs and reports its sample (one frame, after one warm-up frame)."""
    r = bench.cpu_frames(frames=1, warmup=1, prompt=16, cache_len=20, layers=1)
    assert r['frames'] == 1 and r['value'] > 0 and r['cache_len'] == 20 and r['threads'] == bench.cpu_threads()
