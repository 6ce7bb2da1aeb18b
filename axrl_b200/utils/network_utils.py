"""Host networking helpers (reference ``axrl/utils/network_utils.py:22-123``): local IP, free
ports, interface addresses."""

from __future__ import annotations

import socket


def get_free_port(host: str = "127.0.0.1") -> int:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind((host, 0))
        return s.getsockname()[1]


def is_port_free(port: int, host: str = "127.0.0.1") -> bool:
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        try:
            s.bind((host, port))
            return True
        except OSError:
            return False


def get_local_ip() -> str:
    """The address this host would use for outbound traffic (no packet is sent); 127.0.0.1 when
    there is no route."""
    with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
        try:
            s.connect(("10.255.255.255", 1))
            return s.getsockname()[0]
        except OSError:
            return "127.0.0.1"


def interface_addresses() -> dict[str, str]:
    """IPv4 address of every interface (Linux ioctl)."""
    import fcntl
    import struct

    out = {}
    for _, name in socket.if_nameindex():
        with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
            try:
                packed = fcntl.ioctl(s.fileno(), 0x8915, struct.pack("256s", name[:15].encode()))  # SIOCGIFADDR
                out[name] = socket.inet_ntoa(packed[20:24])
            except OSError:
                continue
    return out
