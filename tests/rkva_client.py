"""A minimal RKVA v2 client for the tests of the B200 range server
(xllama-qwen35-xbox_b200/bin/xq_rkva_server): frames requests the way the
reference's host does (RKVA request header + payload) and decodes responses.
Test infrastructure only."""
import os
import socket
import struct
import subprocess

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SERVER = os.path.join(REPO, "xllama-qwen35-xbox_b200", "bin", "xq_rkva_server")

MAGIC, VERSION = 0x41564B52, 2
OP = dict(HELLO=1, CREATE_SESSION=2, DESTROY_SESSION=3, ATTN_DECODE=4, RESET=6, TRIM=7,
          REWIND=8, PING=9, GET_STATS=10, RANGE_CONFIG=12, RANGE_UPLOAD=13, RANGE_ATTN=14,
          KVARN_RANGE_CONFIG=15, RANGE_UPLOAD_ATTN=19)
WIRE = dict(F16=0, F32=1, Q4_0=2, Q8_0=3)
STORAGE = dict(F16=0, Q4_0=1, Q8_0=2)
OK, ERR_PROTOCOL, ERR_UNSUPPORTED_OP, ERR_BAD_SESSION = 0, -1, -2, -3
ERR_BAD_GEOMETRY, ERR_GPU, ERR_BAD_POSITION, ERR_BAD_PAYLOAD, ERR_STATE = -4, -6, -7, -8, -9

REQ = struct.Struct("<IHHQIIII")        # 32 bytes
RSP = struct.Struct("<IHHQiIQQQQ")      # 56 bytes
HELLO = struct.Struct("<16IfQQ")        # 84 bytes
HELLO_ACK = struct.Struct("<4IQQQ")     # 40 bytes
U4 = struct.Struct("<4I")               # session / config / upload / attention headers


def start_server(env=None):
    p = subprocess.Popen([SERVER, "--port", "0", "--once"], stdout=subprocess.PIPE,
                         stderr=subprocess.PIPE, text=True, env=env)
    line = p.stdout.readline()
    assert line.startswith("listening "), line + p.stderr.read()
    return p, int(line.split()[1])


class Client:
    def __init__(self, port):
        self.s = socket.create_connection(("127.0.0.1", port), timeout=60)
        self.s.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self.cycle = 0

    def _recv(self, n):
        buf = b""
        while len(buf) < n:
            chunk = self.s.recv(n - len(buf))
            if not chunk:
                raise ConnectionError("server closed the connection")
            buf += chunk
        return buf

    def call(self, op, payload=b"", session=0, layer=0, n_tokens=0, version=VERSION,
             magic=MAGIC):
        self.cycle += 1
        self.s.sendall(REQ.pack(magic, version, OP.get(op, op) if isinstance(op, str) else op,
                                self.cycle, session, layer, n_tokens, len(payload)) + payload)
        m, ver, rop, cyc, status, nbytes, *_ = RSP.unpack(self._recv(RSP.size))
        assert m == MAGIC and cyc == self.cycle
        return status, self._recv(nbytes) if nbytes else b""

    def hello(self, n_layers, n_head, n_head_kv, head_dim, max_ctx, kq_scale, cache_bits=0):
        fields = [0, n_layers, n_head, n_head_kv, head_dim, max_ctx, cache_bits, cache_bits,
                  0, 0, 0, 0, 0, 0, 0, 0]
        st, body = self.call("HELLO", HELLO.pack(*fields, kq_scale, 0, 0))
        return st, (HELLO_ACK.unpack(body) if st == OK else None)

    def close(self):
        self.s.close()
