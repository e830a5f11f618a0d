// Shared helpers of the two pages: JSON calls, messages, polling, a small line plot.
async function api(path, body) {
  const opt = body === undefined ? {} : {method: "POST", headers: {"Content-Type": "application/json"},
                                         body: JSON.stringify(body)};
  const r = await fetch(path, opt);
  const j = await r.json().catch(() => ({error: `HTTP ${r.status}`}));
  if (!r.ok || j.error) throw new Error(j.error || `HTTP ${r.status}`);
  return j;
}
function $(id) { return document.getElementById(id); }
function say(id, text, bad) { const e = $(id); e.textContent = text; e.className = "msg " + (bad ? "bad" : "ok"); }
function every(ms, fn) { fn(); return setInterval(fn, ms); }
function lines(text) { return text.split("\n").map(s => s.trim()).filter(Boolean); }
function fill(select, names) {
  const cur = select.value;
  select.innerHTML = "<option value=''>(new)</option>" + names.map(n => `<option>${n}</option>`).join("");
  if (names.includes(cur)) select.value = cur;
}
function plot(canvas, xs, ys, label) {
  const dpr = window.devicePixelRatio || 1, w = canvas.clientWidth, h = canvas.clientHeight;
  canvas.width = w * dpr; canvas.height = h * dpr;
  const c = canvas.getContext("2d"); c.scale(dpr, dpr); c.clearRect(0, 0, w, h);
  c.fillStyle = "#6b6b66"; c.font = "11px system-ui"; c.fillText(label, 6, 12);
  if (xs.length < 2) return;
  const x0 = Math.min(...xs), x1 = Math.max(...xs), y0 = Math.min(...ys), y1 = Math.max(...ys);
  const X = x => 30 + (w - 40) * (x - x0) / ((x1 - x0) || 1), Y = y => h - 16 - (h - 34) * (y - y0) / ((y1 - y0) || 1);
  c.strokeStyle = "#2f5d8a"; c.lineWidth = 1.5; c.beginPath();
  xs.forEach((x, i) => i ? c.lineTo(X(x), Y(ys[i])) : c.moveTo(X(x), Y(ys[i]))); c.stroke();
  c.fillText(y1.toPrecision(4), 2, 24); c.fillText(y0.toPrecision(4), 2, h - 4);
}
