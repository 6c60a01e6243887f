"""Container verification (the library's counterpart of Swiftlet's
scripts/verify_container.py), on CPU: the SHA-256 matches hashlib on
known-answer and file inputs; a clean .qpack container verifies; a flipped
byte, a missing file and a manifest size mismatch are each reported; and
delete_corrupt removes the corrupt file and manifest.json as the script does."""
import hashlib
import json
import os

import pytest

import swiftlet_b200 as swl
from conftest import REF_FIXTURES
from swiftlet_b200 import formats


@pytest.mark.parametrize("data", [b"", b"abc", b"a" * 55, b"a" * 56, b"a" * 64, bytes(range(256)) * 4099])
def test_sha256_matches_hashlib(tmp_path, data):
    p = tmp_path / "f.bin"
    p.write_bytes(data)
    assert swl.sha256_file(str(p)) == hashlib.sha256(data).hexdigest()


@pytest.fixture()
def container(tmp_path):
    out = str(tmp_path / "tiny.qpack")
    formats.repack(os.path.join(REF_FIXTURES, "tiny-model-q4"), out)
    formats.write_hashes(out)
    return out


def test_clean_container_verifies(container):
    rep = swl.verify_container(container)
    assert rep["corrupt"] == 0 and rep["missing"] == 0 and rep["ok"] == rep["checked"] >= 4


def test_flipped_byte_is_corrupt_and_deleted_on_request(container):
    p = os.path.join(container, "packed_experts", "layer_03.bin")
    b = bytearray(open(p, "rb").read())
    b[12345] ^= 0x10
    open(p, "wb").write(bytes(b))
    with pytest.raises(swl.SwiftletError) as err:
        swl.verify_container(container)
    assert err.value.code == swl.SWL_ERR_FORMAT
    assert err.value.report["corrupt"] == 1 and err.value.report["first_bad"] == "packed_experts/layer_03.bin"
    assert os.path.exists(p)  # not deleted unless asked
    with pytest.raises(swl.SwiftletError):
        swl.verify_container(container, delete_corrupt=True)
    assert not os.path.exists(p) and not os.path.exists(os.path.join(container, "manifest.json"))


def test_missing_file_and_manifest_size_mismatch(container):
    os.remove(os.path.join(container, "packed_experts", "layer_00.bin"))
    man = json.load(open(os.path.join(container, "manifest.json")))
    man["files"]["model.safetensors"] += 1
    json.dump(man, open(os.path.join(container, "manifest.json"), "w"))
    with pytest.raises(swl.SwiftletError) as err:
        swl.verify_container(container)
    # corrupt: model.safetensors (its size differs from the manifest's) and
    # manifest.json itself (its hash changed with the edit)
    assert err.value.report["missing"] == 1 and err.value.report["corrupt"] == 2


def test_no_hash_list_is_an_io_error(tmp_path):
    with pytest.raises(swl.SwiftletError) as err:
        swl.verify_container(str(tmp_path))
    assert err.value.code == swl.SWL_ERR_IO
