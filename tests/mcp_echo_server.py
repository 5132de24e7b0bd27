"""A minimal MCP server over stdio (JSON-RPC 2.0, one message per line) used by the agent
tests: one tool, ``echo``, that returns its ``text`` argument (``fail: true`` reports an error)."""
import json
import sys


def main():
    for line in sys.stdin:
        try:
            m = json.loads(line)
        except ValueError:
            continue
        if "id" not in m:
            continue  # notifications
        meth = m.get("method")
        if meth == "initialize":
            res = {"protocolVersion": "2024-11-05", "capabilities": {"tools": {}},
                   "serverInfo": {"name": "echo", "version": "1"}}
        elif meth == "tools/list":
            res = {"tools": [{"name": "echo", "description": "Echo text back.",
                              "inputSchema": {"type": "object", "properties": {"text": {"type": "string"},
                                                                               "fail": {"type": "boolean"}},
                                              "required": ["text"]}}]}
        elif meth == "tools/call":
            a = m["params"].get("arguments", {})
            res = {"content": [{"type": "text", "text": "echo: " + a.get("text", "")}], "isError": bool(a.get("fail"))}
        else:
            print(json.dumps({"jsonrpc": "2.0", "id": m["id"], "error": {"code": -32601, "message": "no method"}}),
                  flush=True)
            continue
        print("log line the client must skip", flush=True)
        print(json.dumps({"jsonrpc": "2.0", "id": m["id"], "result": res}), flush=True)


if __name__ == "__main__":
    main()
