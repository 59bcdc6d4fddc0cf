"""A JSON-schema (draft 2020-12) checker for the keywords the reference's report schemas
use: type, required, properties, additionalProperties (false), enum, const, $ref (local),
oneOf, allOf, if/then, minimum, maximum, minLength, pattern, items, minItems.  Test
infrastructure: returns the list of violations as (json-path, message)."""
from __future__ import annotations

import re

_TYPES = {
    "object": lambda v: isinstance(v, dict),
    "array": lambda v: isinstance(v, list),
    "string": lambda v: isinstance(v, str),
    "integer": lambda v: isinstance(v, int) and not isinstance(v, bool),
    "number": lambda v: isinstance(v, (int, float)) and not isinstance(v, bool),
    "boolean": lambda v: isinstance(v, bool),
    "null": lambda v: v is None,
}


def _resolve(root: dict, ref: str) -> dict:
    assert ref.startswith("#/"), ref
    node = root
    for part in ref[2:].split("/"):
        node = node[part]
    return node


def check(instance, schema: dict, root: dict | None = None, path: str = "$") -> list:
    root = root if root is not None else schema
    errors: list = []
    if "$ref" in schema:
        errors += check(instance, _resolve(root, schema["$ref"]), root, path)
    if "type" in schema:
        types = schema["type"] if isinstance(schema["type"], list) else [schema["type"]]
        if not any(_TYPES[t](instance) for t in types):
            errors.append((path, f"type {type(instance).__name__} not in {types}"))
            return errors
    if "const" in schema and instance != schema["const"]:
        errors.append((path, f"{instance!r} != const {schema['const']!r}"))
    if "enum" in schema and instance not in schema["enum"]:
        errors.append((path, f"{instance!r} not in {schema['enum']}"))
    if isinstance(instance, (int, float)) and not isinstance(instance, bool):
        if "minimum" in schema and instance < schema["minimum"]:
            errors.append((path, f"{instance} < minimum {schema['minimum']}"))
        if "maximum" in schema and instance > schema["maximum"]:
            errors.append((path, f"{instance} > maximum {schema['maximum']}"))
    if isinstance(instance, str):
        if "minLength" in schema and len(instance) < schema["minLength"]:
            errors.append((path, f"shorter than {schema['minLength']}"))
        if "pattern" in schema and not re.search(schema["pattern"], instance):
            errors.append((path, f"{instance!r} does not match {schema['pattern']}"))
    if isinstance(instance, dict):
        props = schema.get("properties", {})
        for key in schema.get("required", []):
            if key not in instance:
                errors.append((path, f"missing required {key!r}"))
        if schema.get("additionalProperties") is False:
            for key in instance:
                if key not in props:
                    errors.append((path, f"unexpected property {key!r}"))
        for key, sub in props.items():
            if key in instance:
                errors += check(instance[key], sub, root, f"{path}.{key}")
    if isinstance(instance, list):
        if "minItems" in schema and len(instance) < schema["minItems"]:
            errors.append((path, f"fewer than {schema['minItems']} items"))
        if "items" in schema:
            for i, item in enumerate(instance):
                errors += check(item, schema["items"], root, f"{path}[{i}]")
    for sub in schema.get("allOf", []):
        errors += check(instance, sub, root, path)
    if "oneOf" in schema:
        matches = sum(1 for sub in schema["oneOf"] if not check(instance, sub, root, path))
        if matches != 1:
            errors.append((path, f"matches {matches} of oneOf"))
    if "if" in schema and not check(instance, schema["if"], root, path):
        if "then" in schema:
            errors += check(instance, schema["then"], root, path)
    return errors
