"""Runtime protobuf + gRPC surface built from the .proto files in api/protos.

There is no protoc in this environment, so the .proto text is parsed here
(the subset the schema uses: packages, imports, messages with nested enums,
enums, scalar / message / enum / repeated / map fields, services with
streaming flags) into FileDescriptorProtos, loaded into a descriptor pool, and
message classes are produced by the protobuf runtime. gRPC servers and clients
use generic handlers keyed by "/lake.<Service>/<Method>".

    from lake_b200.api import proto
    pb = proto.messages()                  # namespace of message classes
    req = pb.LookupPrefixRequest(model_id="m")
    proto.add_service(server, "ControlPlaneService", impl)
    stub = proto.Stub(channel, "ControlPlaneService")
"""
from __future__ import annotations

import os
import re
from dataclasses import dataclass
from types import SimpleNamespace

from google.protobuf import descriptor_pb2, descriptor_pool, message_factory

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "protos")
FDP = descriptor_pb2.FieldDescriptorProto
SCALARS = {
    "double": FDP.TYPE_DOUBLE, "float": FDP.TYPE_FLOAT, "int64": FDP.TYPE_INT64, "uint64": FDP.TYPE_UINT64,
    "int32": FDP.TYPE_INT32, "uint32": FDP.TYPE_UINT32, "bool": FDP.TYPE_BOOL, "string": FDP.TYPE_STRING,
    "bytes": FDP.TYPE_BYTES, "sint32": FDP.TYPE_SINT32, "sint64": FDP.TYPE_SINT64, "fixed32": FDP.TYPE_FIXED32,
    "fixed64": FDP.TYPE_FIXED64,
}


@dataclass
class Method:
    name: str
    input: str
    output: str
    client_stream: bool
    server_stream: bool


def _tokens(text: str) -> list[str]:
    text = re.sub(r"//[^\n]*", "", text)
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r'"[^"]*"|[A-Za-z_][\w.]*|\d+|[{}<>;=(),\[\]]', text)


class _Parser:
    def __init__(self, toks):
        self.t = toks
        self.i = 0

    def peek(self):
        return self.t[self.i] if self.i < len(self.t) else None

    def take(self, want=None):
        tok = self.t[self.i]
        if want is not None and tok != want:
            raise SyntaxError(f"expected {want!r}, got {tok!r} at token {self.i}")
        self.i += 1
        return tok

    def skip_statement(self):
        while self.take() != ";":
            pass


def parse_proto(text: str, name: str):
    """Return (FileDescriptorProto, {service: [Method]}) with type names left to resolve."""
    p = _Parser(_tokens(text))
    fd = descriptor_pb2.FileDescriptorProto(name=name, syntax="proto3")
    services: dict[str, list[Method]] = {}
    raw_fields = []  # (field proto, type token, scope path)

    def parse_enum(container, ename):
        e = container.add(name=ename)
        p.take("{")
        while p.peek() != "}":
            if p.peek() in ("option", "reserved"):
                p.skip_statement()
                continue
            vname = p.take()
            p.take("=")
            num = int(p.take())
            e.value.add(name=vname, number=num)
            p.take(";")
        p.take("}")

    def parse_message(container, mname, scope):
        m = container.add(name=mname)
        path = scope + [mname]
        p.take("{")
        while p.peek() != "}":
            tok = p.peek()
            if tok == "enum":
                p.take()
                parse_enum(m.enum_type, p.take())
            elif tok == "message":
                p.take()
                parse_message(m.nested_type, p.take(), path)
            elif tok in ("option", "reserved"):
                p.skip_statement()
            elif tok == "map":
                p.take()
                p.take("<")
                kt = p.take()
                p.take(",")
                vt = p.take()
                p.take(">")
                fname = p.take()
                p.take("=")
                num = int(p.take())
                p.take(";")
                entry = "".join(w.capitalize() for w in fname.split("_")) + "Entry"
                em = m.nested_type.add(name=entry)
                em.options.map_entry = True
                kf = em.field.add(name="key", number=1, label=FDP.LABEL_OPTIONAL)
                vf = em.field.add(name="value", number=2, label=FDP.LABEL_OPTIONAL)
                raw_fields.append((kf, kt, path + [entry]))
                raw_fields.append((vf, vt, path + [entry]))
                f = m.field.add(name=fname, number=num, label=FDP.LABEL_REPEATED, type=FDP.TYPE_MESSAGE)
                f.type_name = "." + ".".join([fd.package] + path + [entry])
            else:
                label = FDP.LABEL_OPTIONAL
                if tok == "repeated":
                    p.take()
                    label = FDP.LABEL_REPEATED
                elif tok == "optional":
                    p.take()
                ftype = p.take()
                fname = p.take()
                p.take("=")
                num = int(p.take())
                if p.peek() == "[":
                    while p.take() != "]":
                        pass
                p.take(";")
                f = m.field.add(name=fname, number=num, label=label)
                raw_fields.append((f, ftype, path))
        p.take("}")

    while p.peek() is not None:
        tok = p.take()
        if tok == "syntax":
            p.skip_statement()
        elif tok == "package":
            fd.package = p.take()
            p.take(";")
        elif tok == "import":
            fd.dependency.append(p.take().strip('"'))
            p.take(";")
        elif tok == "option":
            p.skip_statement()
        elif tok == "message":
            parse_message(fd.message_type, p.take(), [])
        elif tok == "enum":
            parse_enum(fd.enum_type, p.take())
        elif tok == "service":
            sname = p.take()
            methods = []
            p.take("{")
            while p.peek() != "}":
                p.take("rpc")
                mname = p.take()
                p.take("(")
                cs = p.peek() == "stream"
                if cs:
                    p.take()
                itype = p.take()
                p.take(")")
                p.take("returns")
                p.take("(")
                ss = p.peek() == "stream"
                if ss:
                    p.take()
                otype = p.take()
                p.take(")")
                if p.peek() == "{":
                    while p.take() != "}":
                        pass
                else:
                    p.take(";")
                methods.append(Method(mname, itype, otype, cs, ss))
            p.take("}")
            services[sname] = methods
        else:
            raise SyntaxError(f"unexpected token {tok!r}")
    return fd, services, raw_fields


def _build():
    files = {}
    all_types: dict[str, str] = {}  # fully qualified -> "message" | "enum"
    parsed = {}
    for fname in ("schema.proto", "lake.proto"):
        with open(os.path.join(HERE, fname)) as f:
            fd, services, raw = parse_proto(f.read(), fname)
        parsed[fname] = (fd, services, raw)

        def collect(prefix, msgs, enums):
            for e in enums:
                all_types[f"{prefix}.{e.name}"] = "enum"
            for m in msgs:
                all_types[f"{prefix}.{m.name}"] = "message"
                collect(f"{prefix}.{m.name}", m.nested_type, m.enum_type)

        collect(fd.package, fd.message_type, fd.enum_type)

    def resolve(tname, scope, package):
        if tname.startswith("lake.") and tname in all_types:
            return tname
        for i in range(len(scope), -1, -1):
            cand = ".".join([package] + scope[:i] + [tname])
            if cand in all_types:
                return cand
        raise KeyError(f"unknown type {tname} in scope {scope}")

    pool = descriptor_pool.DescriptorPool()
    for fname in ("schema.proto", "lake.proto"):
        fd, services, raw = parsed[fname]
        for f, ftype, scope in raw:
            if ftype in SCALARS:
                f.type = SCALARS[ftype]
            else:
                fq = resolve(ftype, scope, fd.package)
                f.type = FDP.TYPE_MESSAGE if all_types[fq] == "message" else FDP.TYPE_ENUM
                f.type_name = "." + fq
        for sname, methods in services.items():
            sd = fd.service.add(name=sname)
            for mth in methods:
                md = sd.method.add(name=mth.name, input_type="." + resolve(mth.input, [], fd.package),
                                   output_type="." + resolve(mth.output, [], fd.package))
                md.client_streaming = mth.client_stream
                md.server_streaming = mth.server_stream
        pool.Add(fd)
        files[fname] = fd
    classes = {}
    for fq, kind in all_types.items():
        if kind == "message" and fq.count(".") == 1:
            classes[fq.split(".", 1)[1]] = message_factory.GetMessageClass(pool.FindMessageTypeByName(fq))
    enums = {}
    for fq, kind in all_types.items():
        if kind == "enum":
            ed = pool.FindEnumTypeByName(fq)
            enums[fq.split(".", 1)[1]] = {v.name: v.number for v in ed.values}
    services = {}
    for fname in ("schema.proto", "lake.proto"):
        services.update(parsed[fname][1])
    return pool, classes, enums, services


_CACHE = None


def _state():
    global _CACHE
    if _CACHE is None:
        _CACHE = _build()
    return _CACHE


def messages() -> SimpleNamespace:
    """Namespace of message classes (pb.KVBlockID, pb.Ack, ...) and enum value maps (pb.enums)."""
    pool, classes, enums, services = _state()
    ns = SimpleNamespace(**classes)
    ns.enums = enums
    return ns


def services() -> dict[str, list[Method]]:
    return _state()[3]


def _cls(name):
    return _state()[1][name.split(".")[-1]]


def _snake(name: str) -> str:
    return re.sub(r"(?<!^)(?=[A-Z])", "_", name).lower()


def add_service(server, service: str, impl) -> None:
    """Register `impl` (methods named like the rpc, CamelCase or snake_case) on a grpc server."""
    import grpc

    handlers = {}
    for m in services()[service]:
        fn = getattr(impl, m.name, None) or getattr(impl, _snake(m.name), None)
        if fn is None:
            continue
        req, resp = _cls(m.input), _cls(m.output)
        kw = dict(request_deserializer=req.FromString, response_serializer=resp.SerializeToString)
        if m.client_stream and m.server_stream:
            h = grpc.stream_stream_rpc_method_handler(fn, **kw)
        elif m.client_stream:
            h = grpc.stream_unary_rpc_method_handler(fn, **kw)
        elif m.server_stream:
            h = grpc.unary_stream_rpc_method_handler(fn, **kw)
        else:
            h = grpc.unary_unary_rpc_method_handler(fn, **kw)
        handlers[m.name] = h
    server.add_generic_rpc_handlers((grpc.method_handlers_generic_handler(f"lake.{service}", handlers),))


class Stub:
    """Client for one service: stub.LookupPrefix(req) etc."""

    def __init__(self, channel, service: str):
        for m in services()[service]:
            req, resp = _cls(m.input), _cls(m.output)
            path = f"/lake.{service}/{m.name}"
            kw = dict(request_serializer=req.SerializeToString, response_deserializer=resp.FromString)
            if m.client_stream and m.server_stream:
                call = channel.stream_stream(path, **kw)
            elif m.client_stream:
                call = channel.stream_unary(path, **kw)
            elif m.server_stream:
                call = channel.unary_stream(path, **kw)
            else:
                call = channel.unary_unary(path, **kw)
            setattr(self, m.name, call)


MAX_MESSAGE_BYTES = 256 << 20


def message_options() -> list[tuple[str, int]]:
    """gRPC channel/server options for services that carry KV pages (a Llama-3-8B page is
    2 MiB; gRPC's default receive limit is 4 MiB)."""
    return [("grpc.max_send_message_length", MAX_MESSAGE_BYTES),
            ("grpc.max_receive_message_length", MAX_MESSAGE_BYTES)]
