"""Web search and page scraping through the Serper API as an MCP environment (reference
environment: mcp_tools/serper_search/server.py:64-136).

Tools: ``search`` (Google web results), ``search_places`` and ``scrape_webpage`` (page text,
truncated to ``max_scrape_chars``).  Requests are POSTs with the ``X-API-KEY`` header read
from ``SERPER_API_KEY``; failures come back as ``{"error": ...}`` so a rollout can continue.
The HTTP call is injectable (``post``) so the server can be exercised without a network.

    SERPER_API_KEY=... python -m agent_factory_3_b200.envs.serper_search
"""
from __future__ import annotations

import argparse
import os
from typing import Annotated, Any, Awaitable, Callable

SEARCH_URL = "https://google.serper.dev/search"
PLACES_URL = "https://google.serper.dev/places"
SCRAPE_URL = "https://scrape.serper.dev"

Post = Callable[[str, dict, dict], Awaitable[dict]]


async def aiohttp_post(url: str, headers: dict, payload: dict, timeout_s: float = 30.0) -> dict:
    import aiohttp

    async with aiohttp.ClientSession(timeout=aiohttp.ClientTimeout(total=timeout_s)) as s:
        async with s.post(url, headers=headers, json=payload) as r:
            if r.status != 200:
                return {"error": f"HTTP {r.status}: {(await r.text())[:500]}"}
            return await r.json()


def build_server(api_key: str | None = None, post: Post | None = None,
                 max_scrape_chars: int = 20000):
    from mcp.server.fastmcp import FastMCP

    key = api_key if api_key is not None else os.environ.get("SERPER_API_KEY", "")
    post = post or aiohttp_post
    mcp = FastMCP(name="serper_search", instructions=(
        "Web search tools: 'search' returns Google results (title, link, snippet), "
        "'search_places' returns places, 'scrape_webpage' returns the text of a page."))

    async def call(url: str, payload: dict) -> dict[str, Any]:
        if not key:
            return {"error": "SERPER_API_KEY is not set"}
        try:
            return await post(url, {"X-API-KEY": key, "Content-Type": "application/json"}, payload)
        except Exception as e:  # noqa: BLE001 - network errors are tool results, not crashes
            return {"error": f"{type(e).__name__}: {e}"}

    @mcp.tool(description="Search the web. Returns organic results with title, link and snippet.")
    async def search(q: Annotated[str, "search query"],
                     num: Annotated[int, "number of results (1-100)"] = 10,
                     gl: Annotated[str, "country code, e.g. us"] = "us",
                     hl: Annotated[str, "language code, e.g. en"] = "en") -> dict:
        return await call(SEARCH_URL, {"q": q, "num": max(1, min(int(num), 100)), "gl": gl, "hl": hl})

    @mcp.tool(description="Search for places (businesses, landmarks) matching a query.")
    async def search_places(q: Annotated[str, "search query"],
                            gl: Annotated[str, "country code"] = "us",
                            hl: Annotated[str, "language code"] = "en") -> dict:
        return await call(PLACES_URL, {"q": q, "gl": gl, "hl": hl})

    @mcp.tool(description="Fetch a web page and return its text content.")
    async def scrape_webpage(url: Annotated[str, "page URL"]) -> dict:
        r = await call(SCRAPE_URL, {"url": url})
        text = r.get("text")
        if isinstance(text, str) and len(text) > max_scrape_chars:
            r = {**r, "text": text[:max_scrape_chars], "truncated": True}
        return r

    return mcp


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--max-scrape-chars", type=int, default=20000)
    a = ap.parse_args()
    build_server(max_scrape_chars=a.max_scrape_chars).run()


if __name__ == "__main__":
    main()
