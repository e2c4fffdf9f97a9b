"""Inline stylesheet and script of the rollout viewer page (no external assets)."""

CSS = """
:root{--bg:#0f1117;--card:#171a23;--fg:#e6e6e6;--mute:#8a8f98;--acc:#6aa6ff;--ok:#3fb950;
--bad:#f85149;--warn:#d29922;--line:#262a35}
*{box-sizing:border-box}
body{background:var(--bg);color:var(--fg);font:14px/1.45 system-ui,-apple-system,Segoe UI,sans-serif;margin:0}
header{padding:14px 20px;border-bottom:1px solid var(--line);position:sticky;top:0;background:var(--bg);z-index:5}
h1{font-size:19px;margin:0 0 6px}h2{font-size:16px;margin:0 0 8px}h3{font-size:13px;color:var(--mute);margin:16px 0 6px}
.summary{color:var(--mute);margin-bottom:8px}
input#filter{background:var(--card);color:var(--fg);border:1px solid #333;border-radius:6px;padding:5px 10px;width:360px}
main{display:flex;height:calc(100vh - 110px)}
nav#list{width:38%;min-width:320px;overflow-y:auto;padding:12px;border-right:1px solid var(--line)}
section#pane{flex:1;overflow-y:auto;padding:16px 22px}
.empty{color:var(--mute);margin-top:40px;text-align:center}
.group{background:var(--card);border:1px solid var(--line);border-radius:9px;padding:8px 10px;margin-bottom:10px}
.gh{margin-bottom:4px}.meta{color:var(--mute);font-size:11px;margin-bottom:4px;word-break:break-all}
.row{display:flex;gap:8px;align-items:center;padding:3px 6px;border-radius:5px;cursor:pointer;font-size:13px}
.row:hover{background:#1f2430}.row.sel{background:#23304a}.row.skipped{opacity:.6}
.rid{flex:1;overflow:hidden;text-overflow:ellipsis;white-space:nowrap}
.num{color:#c9d1d9;font-variant-numeric:tabular-nums}.num.adv{color:var(--acc)}
.end{color:var(--mute);font-size:11px}
.dot{width:9px;height:9px;border-radius:50%;display:inline-block;background:#555}
.dot.ok{background:var(--ok)}.dot.fail{background:var(--warn)}.dot.bad{background:var(--bad)}
.badge{display:inline-block;border-radius:10px;padding:1px 8px;font-size:12px;margin:0 4px 2px 0;background:#262a35}
.badge.ok{background:#12361f;color:var(--ok)}.badge.bad{background:#3d1618;color:var(--bad)}
.badge.warn{background:#3a2c10;color:var(--warn)}
table.facts{border-collapse:collapse;margin:8px 0}table.facts th{text-align:left;color:var(--mute);
font-weight:500;padding:1px 14px 1px 0}table.facts td{padding:1px 0}
.msg{margin:6px 0;padding:7px 10px;border-radius:6px;background:#1d212c;white-space:pre-wrap;word-break:break-word}
.msg .role{font-size:11px;color:var(--mute);text-transform:uppercase;letter-spacing:.05em;margin-bottom:3px;cursor:default}
details.msg>summary.role{cursor:pointer}
.msg.system,.msg.developer{background:#1a1d26;color:#b8bcc6}
.msg.analysis{border-left:3px solid #555}.msg.commentary{border-left:3px solid var(--warn)}
.msg.final{border-left:3px solid var(--ok)}.msg.tool{border-left:3px solid var(--acc);background:#161b26}
.msg.error{border-left:3px solid var(--bad)}.msg.warn{border-left:3px solid var(--warn)}
.msg.call .role{color:var(--warn)}
details.long>summary{cursor:pointer;color:var(--mute)}
pre{white-space:pre-wrap;font-size:12px;margin:4px 0}
"""

JS = """
(function(){
const rows=[...document.querySelectorAll('.row')];let cur=-1;
function show(i){if(i<0||i>=rows.length)return;if(cur>=0)rows[cur].classList.remove('sel');cur=i;
const r=rows[i];r.classList.add('sel');r.scrollIntoView({block:'nearest'});
const t=document.getElementById(r.dataset.d);const p=document.getElementById('pane');
p.innerHTML='';p.appendChild(t.content.cloneNode(true));p.scrollTop=0;}
rows.forEach((r,i)=>r.addEventListener('click',()=>show(i)));
function visible(i){return rows[i].offsetParent!==null}
document.addEventListener('keydown',e=>{if(e.target.tagName==='INPUT')return;
if(e.key==='j'){let i=cur+1;while(i<rows.length&&!visible(i))i++;show(i)}
if(e.key==='k'){let i=cur-1;while(i>=0&&!visible(i))i--;show(i)}});
document.getElementById('filter').addEventListener('input',e=>{const q=e.target.value.toLowerCase();
document.querySelectorAll('.group').forEach(g=>{const gm=g.querySelector('.gh').innerText.toLowerCase().includes(q);
let any=false;g.querySelectorAll('.row').forEach(r=>{const m=gm||r.innerText.toLowerCase().includes(q);
r.style.display=m?'':'none';any=any||m});g.style.display=any?'':'none'})});
if(rows.length)show(0);
})();
"""
