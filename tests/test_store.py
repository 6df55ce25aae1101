"""Object store: content addressing, manifests, refs (CAS), leases, GC, corruption, crash recovery."""

import hashlib
import os
import subprocess
import sys

import pytest

from reelcache_b200.errors import IntegrityError, QuarantinedError, StateError
from reelcache_b200.store import EvictedObjectError, ObjectStore


def test_content_addressing_and_dedup(tmp_path):
    with ObjectStore(tmp_path / "s") as store:
        a = store.put(b"hello")
        assert a == "blob:" + hashlib.sha256(b"hello").hexdigest()
        assert store.put(b"hello") == a
        assert store.get(a) == b"hello"
        assert (tmp_path / "s" / "objects" / "blob" / a.split(":")[1]).exists()
        assert store.stats()["objects"] == 1


def test_manifest_references_and_gc(tmp_path):
    with ObjectStore(tmp_path / "s") as store:
        blob = store.put(b"payload")
        other = store.put(b"garbage")
        manifest = store.put_manifest({"x": 1}, references=[blob])
        data, refs = store.get_manifest_with_references(manifest)
        assert data == {"x": 1} and refs == (blob,)
        store.set_ref("heads/main", manifest, expected=None)
        result = store.collect_garbage()
        assert result["objects_removed"] == 1
        with pytest.raises(IntegrityError):
            store.get(other)
        assert store.get(blob) == b"payload"


def test_ref_compare_and_swap(tmp_path):
    with ObjectStore(tmp_path / "s") as store:
        a = store.put_manifest({"a": 1})
        b = store.put_manifest({"b": 1})
        store.set_ref("r", a, expected=None)
        with pytest.raises(StateError):
            store.set_ref("r", b, expected=None)
        store.set_ref("r", b, expected=a)
        assert store.get_ref("r") == b
        store.delete_ref("r", expected=b)
        assert store.get_ref("r") is None


def test_lease_pins_until_released(tmp_path):
    with ObjectStore(tmp_path / "s") as store:
        blob = store.put(b"pinned")
        lease = store.lease(blob)
        store.collect_garbage()
        assert store.get(blob) == b"pinned"
        lease.release()
        store.collect_garbage()
        with pytest.raises(IntegrityError):
            store.get(blob)


def test_corruption_detected_and_quarantined(tmp_path):
    with ObjectStore(tmp_path / "s", verify_reads=True) as store:
        blob = store.put(b"original bytes")
        path = store.path_for(blob)
        path.write_bytes(b"original bytez")
        with pytest.raises(IntegrityError):
            store.get(blob)
        assert blob in store.quarantined_objects
        with pytest.raises(QuarantinedError):
            store.get(blob)
        path.write_bytes(b"original bytes")
        assert store.get(blob) == b"original bytes"
        assert blob not in store.quarantined_objects


def test_reopen_and_missing_index_refused(tmp_path):
    root = tmp_path / "s"
    with ObjectStore(root) as store:
        m = store.put_manifest({"k": "v"})
        store.set_ref("r", m)
    with ObjectStore(root) as store:
        assert store.get_manifest(store.get_ref("r")) == {"k": "v"}
    os.remove(root / "index.sqlite3")
    with pytest.raises(IntegrityError):
        ObjectStore(root)


def test_staging_leases_of_dead_process_are_recovered(tmp_path):
    root = tmp_path / "s"
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from reelcache_b200.store import ObjectStore\n"
        "s = ObjectStore(%r)\n"
        "b = s.put(b'staged-by-child')\n"
        "lease = s.lease(b, purpose='staging')\n"
        "import os; os._exit(0)\n" % (os.path.dirname(os.path.dirname(os.path.abspath(__file__))), str(root))
    )
    subprocess.run([sys.executable, "-c", code], check=True)
    with ObjectStore(root) as store:
        assert store.stats()["objects"] == 0


def test_evict_and_restore_by_rewrite(tmp_path):
    with ObjectStore(tmp_path / "s") as store:
        blob = store.put(b"evict me")
        manifest = store.put_manifest({}, references=[blob])
        store.set_ref("r", manifest)
        assert store.evict([blob])["evicted"] == 1
        with pytest.raises(EvictedObjectError):
            store.get(blob)
        store.put(b"evict me")
        assert store.get(blob) == b"evict me"


def test_telemetry_sidecar_not_in_content(tmp_path):
    with ObjectStore(tmp_path / "s") as store:
        m = store.put_manifest({"a": 1})
        store.put_telemetry(m, {"seconds": 1.5})
        assert store.telemetry(m) == {"seconds": 1.5}
        assert store.put_manifest({"a": 1}) == m


def test_reference_updates_walk_only_new_objects(tmp_path):
    """A reference update checks each new object once: a chain of nodes published one after another walks only
    what each node adds (the checked history is not read again), and collection after the updates still keeps
    every reachable object."""
    with ObjectStore(tmp_path / "s") as store:
        head = None
        for i in range(5):
            blob = store.put(f"payload {i}".encode())
            head = store.put_manifest({"i": i}, references=[blob] + ([head] if head else []))
            store.set_ref("heads/main", head)
        reads = []
        original = store._manifest
        store._manifest = lambda object_id: (reads.append(object_id), original(object_id))[1]
        blob = store.put(b"payload 5")
        top = store.put_manifest({"i": 5}, references=[blob, head])
        store.set_ref("heads/main", top)
        store._manifest = original
        assert head not in reads  # the previous head's subtree was checked by the previous update
        assert store.collect_garbage()["live_objects"] == 12
