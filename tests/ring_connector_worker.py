"""Producer process for the cross-process ring-connector GPU tests.

``python tests/ring_connector_worker.py <shared_dir> <device> <seed>``: builds
the seeded paged cache of ``tests/test_ring_connector.py``, saves the chunk
through ``HcpRingKvConnector`` (``save_kv_layer`` per layer, then
``wait_for_save``, which exports the chunk store and writes the marker), then
keeps the store alive until ``<shared_dir>/done`` appears (at most 180 s).
"""

from __future__ import annotations

import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    shared, device, seed = sys.argv[1], int(sys.argv[2]), int(sys.argv[3])
    import torch
    from tests.test_ring_connector import produce

    torch.cuda.set_device(device)
    conn = produce(shared, torch.device("cuda", device), seed)
    t0 = time.time()
    while not os.path.exists(os.path.join(shared, "done")) and time.time() - t0 < 180:
        time.sleep(0.05)
    conn.shutdown()
    return 0


if __name__ == "__main__":
    sys.exit(main())
