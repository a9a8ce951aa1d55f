"""The decode driver's CPU SIEVE checker (kv_offload_proto_b200.decode.SieveChecker, the
reference driver's model xds_decode.py:66-118) against the C restatement on the same inputs,
and the driver's option parsing. The driver itself runs on the GPU (test_gpu_decode_driver)."""
import numpy as np

import oracle
from kv_offload_proto_b200.decode import SieveChecker, parse_args
from kv_offload_proto_b200.workload import ref_topk_batch


def test_checker_equals_the_c_restatement():
    rng = np.random.default_rng(3)
    for R, prefill, dbs, K, miss in ((8, 256, 64, 64, 0.5), (3, 500, 128, 100, 0.3), (2, 64, 64, 32, 0.5)):
        st = oracle.SieveState(1, R, dbs, K)
        ck = SieveChecker()
        for r in range(R):
            st.admit(r, prefill)
            ck.reset(r, prefill, dbs)
        for _ in range(12):
            batch = ref_topk_batch(rng, R, K, prefill, dbs, miss)
            batch[0, :3] = [-1, prefill + 2, prefill - 1]  # invalid, decode-extension, last prefill token
            seq = np.full(R, prefill + 4, np.int32)
            exp_slots, exp_miss = st.update(0, batch, np.arange(R), seq)
            for r in range(R):
                s, m = ck.update(r, batch[r], int(seq[r]), st.padded)
                np.testing.assert_array_equal(np.array(s, np.int32), exp_slots[r])
                np.testing.assert_array_equal(np.array(m, np.int8), exp_miss[r])


def test_driver_options_keep_the_reference_names_and_defaults():
    a = parse_args([])
    assert (a.layers, a.layer_rows, a.kv_lora_rank, a.qk_rope, a.stripe_rows, a.req_num, a.prefill, a.topk,
            a.device_buffer_size, a.miss_ratio, a.steps, a.seed, a.block_dim) == \
        (2, 1024, 512, 64, 1, 8, 256, 64, 64, 0.5, 10, 42, 8)  # xds_decode.py:21-45
    assert not a.oracle and a.run_dir == "./log"
