"""Agent tooling: a tool registry with built-in tools, an MCP client, and the tool-calling loop."""
