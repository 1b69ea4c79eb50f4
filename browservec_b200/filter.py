"""Metadata predicates with the reference's semantics (src/store/filter.ts:18-68).

``compile_filter`` turns a Mongo-ish filter into a predicate over one record's
metadata dict; ``FilterColumns`` evaluates the same predicate over a whole
store at once (dictionary-coded columns, numpy), which is what the mask of a
filtered query is built from (src/index.ts:372-395).

JavaScript equality is strict (===): a bool never equals a number, ``None``
(null) never equals a missing field (undefined), and numbers compare by value
(1 === 1.0).  ``$in`` tests membership with ``Set.has`` (filter.ts:29-30),
whose SameValueZero also matches NaN to NaN.  Range operators match stored
numbers only.
"""
from __future__ import annotations

import ctypes as C
from typing import Any, Callable, Mapping

import numpy as np

OPS = ("$eq", "$ne", "$in", "$gt", "$gte", "$lt", "$lte")
_MISSING = object()  # JS undefined


def _is_number(v: Any) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool)


def strict_eq(a: Any, b: Any) -> bool:
    """JS `a === b` for metadata values (string | number | boolean | null | undefined)."""
    if a is _MISSING or b is _MISSING:
        return a is b
    if a is None or b is None:
        return a is None and b is None
    if isinstance(a, bool) or isinstance(b, bool):
        return isinstance(a, bool) and isinstance(b, bool) and a == b
    if _is_number(a) and _is_number(b):
        return float(a) == float(b)
    if isinstance(a, str) and isinstance(b, str):
        return a == b
    return False


def same_value_zero(a: Any, b: Any) -> bool:
    """JS SameValueZero (Set.has): === except that NaN equals NaN."""
    if _is_number(a) and _is_number(b) and a != a and b != b:
        return True
    return strict_eq(a, b)


def _get(m: Mapping | None, field: str) -> Any:
    if m is None:
        return _MISSING
    return m.get(field, _MISSING)


def _compile_op(field: str, op: str, arg: Any) -> Callable[[Mapping | None], bool]:
    """filter.ts:35-66"""
    if op == "$eq":
        return lambda m: strict_eq(_get(m, field), arg)
    if op == "$ne":  # also matches records missing the field
        return lambda m: not strict_eq(_get(m, field), arg)
    if op == "$in":
        if not isinstance(arg, (list, tuple)):
            raise ValueError(f'filter: $in on "{field}" expects an array, got {_js_typeof(arg)}')
        vals = list(arg)
        return lambda m: any(same_value_zero(_get(m, field), v) for v in vals)
    if op in ("$gt", "$gte", "$lt", "$lte"):
        if not _is_number(arg):
            raise ValueError(f'filter: {op} on "{field}" expects a number, got {_js_typeof(arg)}')
        cmp = {"$gt": lambda v: v > arg, "$gte": lambda v: v >= arg,
               "$lt": lambda v: v < arg, "$lte": lambda v: v <= arg}[op]
        return lambda m: _is_number(_get(m, field)) and cmp(_get(m, field))
    raise ValueError(f'filter: unknown operator "{op}" on field "{field}"')


def _js_typeof(v: Any) -> str:
    if v is None:
        return "object"
    if isinstance(v, bool):
        return "boolean"
    if _is_number(v):
        return "number"
    if isinstance(v, str):
        return "string"
    return "object"


def _is_ops(cond: Any) -> bool:
    return isinstance(cond, Mapping)


def compile_filter(flt: Mapping[str, Any]) -> Callable[[Mapping | None], bool]:
    """filter.ts:52-68: AND across fields and operators; a bare value is $eq."""
    tests = []
    for field, cond in flt.items():
        if _is_ops(cond):
            for op, arg in cond.items():
                if op not in OPS:
                    raise ValueError(f'filter: unknown operator "{op}" on field "{field}"')
                tests.append(_compile_op(field, op, arg))
        else:
            tests.append(_compile_op(field, "$eq", cond))
    return lambda m: all(t(m) for t in tests)


class FilterColumns:
    """Column store of per-row metadata for vectorised predicate evaluation.

    Each field is kept as a numeric column (float64, NaN where the value is
    not a number), a type-tag column and, for strings, dictionary codes.
    ``mask(filter)`` returns the same bit set the row loop of
    src/index.ts:372-386 builds, as 1 bit per row in uint32 words.
    """

    T_MISSING, T_NULL, T_BOOL, T_NUM, T_STR = range(5)

    def __init__(self):
        self.n = 0
        self.cols: dict[str, dict] = {}

    def _col(self, field: str) -> dict:
        c = self.cols.get(field)
        if c is None:
            c = {"tag": np.zeros(self.n, np.uint8), "num": np.full(self.n, np.nan),
                 "code": np.full(self.n, -1, np.int64), "dict": {}}
            self.cols[field] = c
        return c

    def append(self, metas: list[Mapping | None]) -> None:
        m = len(metas)
        for c in self.cols.values():
            c["tag"] = np.concatenate([c["tag"], np.zeros(m, np.uint8)])
            c["num"] = np.concatenate([c["num"], np.full(m, np.nan)])
            c["code"] = np.concatenate([c["code"], np.full(m, -1, np.int64)])
        base = self.n
        self.n += m
        for i, md in enumerate(metas):
            if not md:
                continue
            for field, v in md.items():
                c = self._col(field)
                if len(c["tag"]) < self.n:  # column created now
                    c["tag"] = np.zeros(self.n, np.uint8)
                    c["num"] = np.full(self.n, np.nan)
                    c["code"] = np.full(self.n, -1, np.int64)
                r = base + i
                if v is None:
                    c["tag"][r] = self.T_NULL
                elif isinstance(v, bool):
                    c["tag"][r] = self.T_BOOL
                    c["num"][r] = 1.0 if v else 0.0
                elif _is_number(v):
                    c["tag"][r] = self.T_NUM
                    c["num"][r] = float(v)
                elif isinstance(v, str):
                    c["tag"][r] = self.T_STR
                    c["code"][r] = c["dict"].setdefault(v, len(c["dict"]))

    def append_columns(self, count: int, columns: Mapping[str, np.ndarray],
                       dictionaries: Mapping[str, list] | None = None) -> None:
        """Bulk append: numeric columns (all rows numbers) or string columns given
        as integer codes into ``dictionaries[field]``."""
        dictionaries = dictionaries or {}
        for c in self.cols.values():
            c["tag"] = np.concatenate([c["tag"], np.zeros(count, np.uint8)])
            c["num"] = np.concatenate([c["num"], np.full(count, np.nan)])
            c["code"] = np.concatenate([c["code"], np.full(count, -1, np.int64)])
        base = self.n
        self.n += count
        for field, arr in columns.items():
            c = self._col(field)
            if len(c["tag"]) < self.n:
                c["tag"] = np.zeros(self.n, np.uint8)
                c["num"] = np.full(self.n, np.nan)
                c["code"] = np.full(self.n, -1, np.int64)
            arr = np.asarray(arr)
            if field in dictionaries:
                words = list(dictionaries[field])
                remap = np.array([c["dict"].setdefault(w, len(c["dict"])) for w in words], np.int64)
                c["tag"][base:] = self.T_STR
                c["code"][base:] = remap[arr.astype(np.int64)]
            else:
                c["tag"][base:] = self.T_NUM
                c["num"][base:] = arr.astype(np.float64)

    def _eq(self, field: str, arg: Any) -> np.ndarray:
        c = self.cols.get(field)
        if c is None:
            return np.zeros(self.n, bool)
        tag = c["tag"]
        if arg is None:
            return tag == self.T_NULL
        if isinstance(arg, bool):
            return (tag == self.T_BOOL) & (c["num"] == (1.0 if arg else 0.0))
        if _is_number(arg):
            return (tag == self.T_NUM) & (c["num"] == float(arg))
        if isinstance(arg, str):
            code = c["dict"].get(arg)
            return np.zeros(self.n, bool) if code is None else (tag == self.T_STR) & (c["code"] == code)
        return np.zeros(self.n, bool)

    def _op(self, field: str, op: str, arg: Any) -> np.ndarray:
        if op == "$eq":
            return self._eq(field, arg)
        if op == "$ne":
            return ~self._eq(field, arg)
        if op == "$in":
            if not isinstance(arg, (list, tuple)):
                raise ValueError(f'filter: $in on "{field}" expects an array, got {_js_typeof(arg)}')
            out = np.zeros(self.n, bool)
            for v in arg:
                if _is_number(v) and v != v:  # SameValueZero: NaN finds stored NaN
                    c = self.cols.get(field)
                    if c is not None:
                        out |= (c["tag"] == self.T_NUM) & np.isnan(c["num"])
                else:
                    out |= self._eq(field, v)
            return out
        if op in ("$gt", "$gte", "$lt", "$lte"):
            if not _is_number(arg):
                raise ValueError(f'filter: {op} on "{field}" expects a number, got {_js_typeof(arg)}')
            c = self.cols.get(field)
            if c is None:
                return np.zeros(self.n, bool)
            num = np.where(c["tag"] == self.T_NUM, c["num"], np.nan)
            with np.errstate(invalid="ignore"):
                return {"$gt": num > arg, "$gte": num >= arg, "$lt": num < arg, "$lte": num <= arg}[op]
        raise ValueError(f'filter: unknown operator "{op}" on field "{field}"')

    def match(self, flt: Mapping[str, Any]) -> np.ndarray:
        out = np.ones(self.n, bool)
        for field, cond in flt.items():
            if _is_ops(cond):
                for op, arg in cond.items():
                    if op not in OPS:
                        raise ValueError(f'filter: unknown operator "{op}" on field "{field}"')
                    out &= self._op(field, op, arg)
            else:
                out &= self._eq(field, cond)
        return out


def pack_mask(bits: np.ndarray) -> np.ndarray:
    """bool[n] -> uint32[ceil(n/32)] with bit r of word r>>5 = bits[r] (LSB first)."""
    n = bits.size
    words = max((n + 31) // 32, 1)
    b = np.zeros(words * 32, np.uint8)
    b[:n] = bits
    return np.packbits(b, bitorder="little").view(np.uint32).copy()


class DeviceColumns:
    """Metadata columns on the GPU, evaluated by the library's predicate kernel
    (bv_filter_mask): per field a type tag (uint8, FilterColumns.T_*), the
    value as f64 (numbers, booleans as 0/1) and string dictionary codes."""

    def __init__(self, device):
        import torch

        self.torch = torch
        self.device = device
        self.n = 0
        self.fields: dict[str, dict] = {}

    @classmethod
    def from_host(cls, fc: FilterColumns, device) -> "DeviceColumns":
        import torch

        dc = cls(device)
        dc.n = fc.n
        for field, c in fc.cols.items():
            dc.fields[field] = {
                "tag": torch.from_numpy(np.ascontiguousarray(c["tag"], np.uint8)).to(device),
                "num": torch.from_numpy(np.ascontiguousarray(c["num"], np.float64)).to(device),
                "code": torch.from_numpy(np.ascontiguousarray(c["code"], np.int64).astype(np.int32)).to(device),
                "dict": dict(c["dict"]),
            }
        return dc

    def set_number_column(self, field: str, values) -> None:
        """A field every row holds as a number (values: a device tensor)."""
        torch = self.torch
        v = values.to(self.device, torch.float64).contiguous()
        self.n = v.numel()
        self.fields[field] = {"tag": torch.full((self.n,), FilterColumns.T_NUM, dtype=torch.uint8, device=self.device),
                              "num": v, "code": None, "dict": {}}

    def set_string_column(self, field: str, codes, dictionary: list) -> None:
        """A field every row holds as a string: codes (device tensor) index `dictionary`."""
        torch = self.torch
        c = codes.to(self.device, torch.int32).contiguous()
        self.n = c.numel()
        self.fields[field] = {"tag": torch.full((self.n,), FilterColumns.T_STR, dtype=torch.uint8, device=self.device),
                              "num": None, "code": c, "dict": {w: i for i, w in enumerate(dictionary)}}

    def _value(self, field: str, v) -> "_lib.BvValue":
        from . import _lib

        if v is None:
            return _lib.BvValue(tag=_lib.TAG_NULL, code=-1, num=0.0)
        if isinstance(v, bool):
            return _lib.BvValue(tag=_lib.TAG_BOOL, code=-1, num=1.0 if v else 0.0)
        if _is_number(v):
            return _lib.BvValue(tag=_lib.TAG_NUMBER, code=-1, num=float(v))
        if isinstance(v, str):
            return _lib.BvValue(tag=_lib.TAG_STRING, code=self.fields[field]["dict"].get(v, -1), num=0.0)
        return _lib.BvValue(tag=_lib.TAG_MISSING + 99, code=-1, num=0.0)  # objects never match

    def units(self, flt: Mapping[str, Any]):
        """The reference filter as (field, op, values) tests over present
        fields, and whether it can match nothing at all.  Raises the
        reference's errors (filter.ts:18-68)."""
        out, never = [], False
        for field, cond in flt.items():
            ops = cond.items() if _is_ops(cond) else [("$eq", cond)]
            for op, arg in ops:
                if op not in OPS:
                    raise ValueError(f'filter: unknown operator "{op}" on field "{field}"')
                if op == "$in" and not isinstance(arg, (list, tuple)):
                    raise ValueError(f'filter: $in on "{field}" expects an array, got {_js_typeof(arg)}')
                if op in ("$gt", "$gte", "$lt", "$lte") and not _is_number(arg):
                    raise ValueError(f'filter: {op} on "{field}" expects a number, got {_js_typeof(arg)}')
                if field not in self.fields:  # no row has the field: only $ne holds
                    never |= op != "$ne"
                    continue
                vals = list(arg) if op == "$in" else [arg]
                bad = [v for v in vals if not (v is None or isinstance(v, (bool, int, float, str)))]
                if bad:  # objects and arrays never equal a stored value
                    if op == "$ne":
                        continue
                    vals = [v for v in vals if not any(v is b for b in bad)]
                if not vals:
                    never = True
                    continue
                out.append((field, op, vals))
        return out, never

    def _launch(self, tests, live, out, stream: int) -> None:
        """One bv_filter_mask call: the AND of at most FILTER_MAX_TERMS tests,
        each with at most FILTER_MAX_IN values."""
        from . import _lib

        names = []
        terms = (_lib.BvFilterTerm * max(1, len(tests)))()
        for t, (field, op, vals) in enumerate(tests):
            if field not in names:
                names.append(field)
            terms[t] = _lib.BvFilterTerm(column=names.index(field), op=_lib.OP_CODES[op], nvals=len(vals))
            for i, v in enumerate(vals):
                terms[t].vals[i] = self._value(field, v)
        cols = (_lib.BvColumn * max(1, len(names)))()
        for i, f in enumerate(names):
            c = self.fields[f]
            cols[i] = _lib.BvColumn(tag=c["tag"].data_ptr(), num=None if c["num"] is None else c["num"].data_ptr(),
                                    code=None if c["code"] is None else c["code"].data_ptr())
        L = _lib.load()
        _lib.check(L.bv_filter_mask(cols, len(names), terms, len(tests), self.n,
                                    C.c_void_p(live.data_ptr()) if live is not None else None,
                                    C.c_void_p(out.data_ptr()), C.c_void_p(stream)))

    def mask(self, flt: Mapping[str, Any], live=None, stream: int = 0):
        """uint32 mask words (a device tensor) of the rows the filter keeps,
        ANDed with `live` (tombstones cleared) when given.  The library call
        takes at most FILTER_MAX_TERMS tests of at most FILTER_MAX_IN values;
        larger filters are evaluated as several calls whose masks are ANDed
        (more tests) or ORed (a longer $in list), so no limit reaches the user."""
        from . import _lib

        torch = self.torch
        words = max((self.n + 31) // 32, 1)
        out = torch.zeros(words, dtype=torch.int32, device=self.device)
        tests, never = self.units(flt)
        if never or self.n == 0:
            return out
        small = [t for t in tests if len(t[2]) <= _lib.FILTER_MAX_IN]
        big = [t for t in tests if len(t[2]) > _lib.FILTER_MAX_IN]
        first = True
        for g in range(0, max(len(small), 1), _lib.FILTER_MAX_TERMS):
            grp = small[g:g + _lib.FILTER_MAX_TERMS]
            if not grp and small:
                break
            dst = out if first else torch.empty_like(out)
            if grp:
                self._launch(grp, live, dst, stream)
            elif live is not None:
                dst.copy_(live[:words])
            else:
                dst.fill_(-1)
            if not first:
                out &= dst
            first = False
        for field, op, vals in big:  # a long $in: OR of its chunks
            acc = torch.zeros_like(out)
            part = torch.empty_like(out)
            for c0 in range(0, len(vals), _lib.FILTER_MAX_IN):
                self._launch([(field, op, vals[c0:c0 + _lib.FILTER_MAX_IN])], live, part, stream)
                acc |= part
            out &= acc
        if self.n % 32:  # bits past the last row stay clear
            out[-1] &= (1 << (self.n % 32)) - 1
        return out
        L = _lib.load()
        _lib.check(L.bv_filter_mask(cols, ncols, terms, nterms, self.n,
                                    C.c_void_p(live.data_ptr()) if live is not None else None,
                                    C.c_void_p(out.data_ptr()), C.c_void_p(stream)))
        return out
