"""Checkpoints of the Llama-3.1-8B geometry: a seeded-weights writer and the
parallel safetensors reader of the weight stores.

The reference loads a local Hugging Face checkpoint (``tools/run_llama31.py``:
``AutoConfig`` / ``AutoTokenizer`` / ``store.load_checkpoint``,
``weight_store.py:109-171``) and there is no real checkpoint or network here,
so :func:`write_seeded_checkpoint` writes the benchmark's seeded random-init
model (the bits of ``BaseWeightStore.fill_seeded``) as a sharded safetensors
checkpoint with an index, a ``config.json`` that ``AutoConfig`` reads as the
Llama-3.1-8B architecture, and a byte-level tokenizer stand-in (256 byte
tokens, reserved fillers, ``<|begin_of_text|>`` = 128000 prepended,
``<|end_of_text|>`` = 128001) that ``AutoTokenizer`` loads, so the
reference's CLI runs unchanged on it.

:func:`load_safetensors_into` is the loader fast path: it parses each
file's header once and reads every BF16 tensor's bytes straight into its
arena view with parallel ``pread`` (``cb_read_file_ranges``, native
threads); other dtypes are read the same way and converted.
"""

import ctypes
import json
import struct
from pathlib import Path

import torch

from . import _native

_DTYPES = {"BF16": (torch.bfloat16, 2), "F16": (torch.float16, 2), "F32": (torch.float32, 4)}
_NAMES = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32"}

BOS_ID = 128000
EOS_ID = 128001
VOCAB = 128256


# ------------------------------------------------------------------ reading
def read_safetensors_header(path):
    """(header dict, byte offset of the data section) of a safetensors file."""

    with open(path, "rb") as source:
        size = struct.unpack("<Q", source.read(8))[0]
        header = json.loads(source.read(size).decode("utf-8"))
    return header, 8 + size


def load_safetensors_into(files, targets, threads=0):
    """Read tensors into preallocated CPU tensors.

    ``files``: {key: path} (``None`` values skipped); ``targets``: {key:
    contiguous CPU tensor}. Returns the set of keys loaded. Shapes must match;
    BF16 data lands directly in the target, other dtypes are converted.
    """

    by_file = {}
    for key, path in files.items():
        if path is not None and key in targets:
            by_file.setdefault(str(path), []).append(key)
    lib = _native.lib()
    loaded = set()
    for path, keys in sorted(by_file.items()):
        header, base = read_safetensors_header(path)
        offsets, dsts, sizes, converts = [], [], [], []
        for key in keys:
            entry = header.get(key)
            if entry is None:
                continue
            target = targets[key]
            if tuple(entry["shape"]) != tuple(target.shape):
                raise ValueError("{} shape {} != expected {}".format(key, tuple(entry["shape"]), tuple(target.shape)))
            begin, end = entry["data_offsets"]
            dtype, width = _DTYPES.get(entry["dtype"], (None, 0))
            if dtype is None:
                raise ValueError("{}: unsupported dtype {}".format(key, entry["dtype"]))
            if end - begin != target.numel() * width:
                raise ValueError("{}: {} data bytes for {} elements".format(key, end - begin, target.numel()))
            if not target.is_contiguous() or target.device.type != "cpu":
                raise ValueError("{}: target must be a contiguous CPU tensor".format(key))
            if dtype == target.dtype:
                dst = target
            else:
                dst = torch.empty(target.shape, dtype=dtype)
                converts.append((target, dst))
            offsets.append(base + begin)
            dsts.append(dst.data_ptr())
            sizes.append(end - begin)
            loaded.add(key)
        if not offsets:
            continue
        n = len(offsets)
        _native.check(
            lib.cb_read_file_ranges(
                path.encode(), n, (ctypes.c_int64 * n)(*offsets), (ctypes.c_void_p * n)(*dsts),
                (ctypes.c_int64 * n)(*sizes), int(threads),
            ),
            "cb_read_file_ranges",
        )
        for target, source in converts:
            target.copy_(source.to(target.dtype))
    return loaded


# ------------------------------------------------------------------ writing
def write_safetensors(path, entries):
    """Stream a safetensors file: ``entries`` = [(key, shape, torch dtype,
    producer)], each producer returning the tensor's CPU data when called
    (one tensor in host memory at a time)."""

    header, offset = {"__metadata__": {"format": "pt"}}, 0
    for key, shape, dtype, _ in entries:
        nbytes = _DTYPES[_NAMES[dtype]][1]
        for d in shape:
            nbytes *= int(d)
        header[key] = {"dtype": _NAMES[dtype], "shape": [int(d) for d in shape], "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    blob = json.dumps(header, separators=(",", ":")).encode("utf-8")
    blob += b" " * (-len(blob) % 8)  # the data section starts 8-byte aligned
    with open(path, "wb") as sink:
        sink.write(struct.pack("<Q", len(blob)))
        sink.write(blob)
        for key, shape, dtype, producer in entries:
            tensor = producer().contiguous()
            if tuple(tensor.shape) != tuple(int(d) for d in shape) or tensor.dtype != dtype:
                raise ValueError("{}: producer returned {} {}".format(key, tuple(tensor.shape), tensor.dtype))
            sink.write(memoryview(tensor.view(torch.uint8).numpy()))


def llama31_8b_config_dict():
    """``config.json`` of the Llama-3.1-8B architecture (untied head)."""

    return {
        "architectures": ["LlamaForCausalLM"],
        "model_type": "llama",
        "hidden_size": 4096,
        "intermediate_size": 14336,
        "num_hidden_layers": 32,
        "num_attention_heads": 32,
        "num_key_value_heads": 8,
        "head_dim": 128,
        "hidden_act": "silu",
        "vocab_size": VOCAB,
        "max_position_embeddings": 131072,
        "rms_norm_eps": 1e-5,
        "rope_theta": 500000.0,
        "rope_scaling": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                         "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
        "attention_bias": False,
        "mlp_bias": False,
        "tie_word_embeddings": False,
        "bos_token_id": BOS_ID,
        "eos_token_id": EOS_ID,
        "torch_dtype": "bfloat16",
    }


def _byte_alphabet():
    """Byte -> printable character of the byte-level BPE convention: bytes
    that are printable Latin-1 map to themselves, the other 68 to the
    characters from U+0100 upwards, in byte order."""

    printable = set(range(ord("!"), ord("~") + 1)) | set(range(0xA1, 0xAC + 1)) | set(range(0xAE, 0xFF + 1))
    table, extra = {}, 0
    for b in range(256):
        if b in printable:
            table[b] = chr(b)
        else:
            table[b] = chr(256 + extra)
            extra += 1
    return table


def write_tokenizer(out_dir):
    """A byte-level tokenizer stand-in over the 128,256-entry vocabulary: ids
    0..255 are the bytes, 128000/128001 begin/end of text, the rest reserved
    fillers; encoding prepends ``<|begin_of_text|>``."""

    from tokenizers import AddedToken, Tokenizer, decoders, models, pre_tokenizers, processors

    alphabet = _byte_alphabet()
    vocab = {alphabet[b]: b for b in range(256)}
    for i in range(256, VOCAB):
        if i == BOS_ID:
            vocab["<|begin_of_text|>"] = i
        elif i == EOS_ID:
            vocab["<|end_of_text|>"] = i
        elif i > EOS_ID:
            vocab["<|reserved_special_token_{}|>".format(i - EOS_ID - 1)] = i
        else:
            vocab["<|reserved_{}|>".format(i)] = i
    tokenizer = Tokenizer(models.BPE(vocab=vocab, merges=[]))
    tokenizer.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)
    tokenizer.decoder = decoders.ByteLevel()
    tokenizer.add_special_tokens([AddedToken("<|begin_of_text|>", special=True),
                                  AddedToken("<|end_of_text|>", special=True)])
    tokenizer.post_processor = processors.TemplateProcessing(
        single="<|begin_of_text|> $A", pair="<|begin_of_text|> $A <|begin_of_text|> $B",
        special_tokens=[("<|begin_of_text|>", BOS_ID)],
    )
    out_dir = Path(out_dir)
    tokenizer.save(str(out_dir / "tokenizer.json"))
    (out_dir / "tokenizer_config.json").write_text(json.dumps({
        "tokenizer_class": "PreTrainedTokenizerFast",
        "bos_token": "<|begin_of_text|>",
        "eos_token": "<|end_of_text|>",
        "model_max_length": 131072,
        "clean_up_tokenization_spaces": False,
    }, indent=1), encoding="utf-8")


def write_seeded_checkpoint(out_dir, seed=0, std=0.02, shard_bytes=5 << 30, device="cuda:0", plan=None):
    """Write the seeded random-init model (the bits of
    ``BaseWeightStore.fill_seeded(seed, std)``) as a sharded safetensors
    checkpoint with ``model.safetensors.index.json``, ``config.json`` and the
    tokenizer stand-in. Tensors are generated one at a time on ``device``."""

    from . import ops
    from .plan import build_llama31_8b_plan
    from .weight_store import is_norm

    plan = plan or build_llama31_8b_plan("matrix_group")
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    keys = sorted(k for k, s in plan.tensors.items() if s.alias_of is None)
    device = torch.device(device)

    def producer(key, shape):
        def make():
            with torch.cuda.device(device), torch.inference_mode():
                t = torch.empty(shape, dtype=torch.bfloat16, device=device)
                if is_norm(key):
                    t.fill_(1.0)
                else:
                    ops.fill_normal_(t, _native.stream_key(seed, key), std=std)
                return t.cpu()
        return make

    shards, current, size = [], [], 0
    for key in keys:
        shape = tuple(plan.tensors[key].shape)
        nbytes = 2
        for d in shape:
            nbytes *= d
        if current and size + nbytes > shard_bytes:
            shards.append(current)
            current, size = [], 0
        current.append((key, shape, torch.bfloat16, producer(key, shape)))
        size += nbytes
    if current:
        shards.append(current)
    weight_map, total = {}, 0
    for i, entries in enumerate(shards):
        name = "model-{:05d}-of-{:05d}.safetensors".format(i + 1, len(shards))
        write_safetensors(out_dir / name, entries)
        for key, shape, _, _ in entries:
            weight_map[key] = name
            n = 2
            for d in shape:
                n *= d
            total += n
    (out_dir / "model.safetensors.index.json").write_text(
        json.dumps({"metadata": {"total_size": total}, "weight_map": weight_map}, indent=1), encoding="utf-8")
    (out_dir / "config.json").write_text(json.dumps(llama31_8b_config_dict(), indent=1), encoding="utf-8")
    write_tokenizer(out_dir)
    return out_dir
